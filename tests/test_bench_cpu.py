"""bench.py's JSON contract where it runs without a GPU: the --impl reference arm
(the reference's FP32 CPU path on the host cores), its rank handling, the
argument checks, and the config dicts both arms print."""

import importlib
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _run(*args, env=None, timeout=300):
    full_env = dict(os.environ, **(env or {}))
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO,
                          env=full_env, capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    proc = _run("--impl", "reference", "--workload", "rmsnorm", "--secondary", "none",
                "--steps", "3", "--warmup", "3")
    assert proc.returncode == 0, proc.stderr
    lines = [l for l in proc.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e", "impl"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == "GB/s" and line["value"] > 0
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 3, 3)
    assert line["higher_is_better"] is True and line["vs_baseline"] is None
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"]
    assert "worker.py:73-74" in base["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"] == "rmsnorm_bf16_4096x4096_eps1e-6"


def test_reference_arm_other_ranks_print_nothing():
    proc = _run("--impl", "reference", "--workload", "rmsnorm", "--secondary", "none",
                "--steps", "3", "--warmup", "3", "--gpus", "2",
                env={"RANK": "1", "WORLD_SIZE": "2"})
    assert proc.returncode == 0, proc.stderr
    assert proc.stdout.strip() == ""


@pytest.mark.parametrize("args", [("--warmup", "2"), ("--steps", "0")])
def test_argument_checks(args):
    proc = _run("--impl", "reference", "--secondary", "none", *args)
    assert proc.returncode != 0


def test_config_dicts_are_shared_and_cpu_only():
    """Both arms print CONFIGS[name](world): computed from sizes alone."""
    bench = importlib.import_module("bench")
    for name, fn in bench.CONFIGS.items():
        for world in (1, 2, 8):
            cfg = fn(world)
            assert isinstance(cfg, dict) and cfg.get("workload"), name
            json.dumps(cfg)
    assert set(bench.CONFIGS) <= set(bench.WORKLOADS)
    assert set(bench.SCALING) >= set(bench.CONFIGS)
