"""The reference's own plumbing drives the sm_100a kernels on the GPU.

The reference package (baseline/_ref, or $BOKT_REFERENCE_PATH) is copied with
its three kernels, search space and legality module replaced by one-line
re-exports of this package (flashattentionanycard_b200.dropin); everything
else runs unmodified:

* its GPU correctness tests (tests/test_correctness.py -m gpu: every smoke
  configuration x seeds x shapes against its FP32 gate, its CUDA-graph
  measurement, its paired confirmation of candidate vs torch baseline);
* its command line (run_benchmark --mode tune --method grid), which runs
  engine.run_search with one fresh `python -m bo_kernel_tuner.tuner.worker`
  process per trial and reads compiled.metadata.shared / n_regs / n_spills
  from what our launch() returns.

Optuna is absent from this image, so the engine runs on the test stand-in in
tests/dropin_stubs (grid order; no TPE).
"""

import json
import subprocess
import sys

import pytest

from flashattentionanycard_b200 import dropin
from tests.dropin import overlay_env, reference_root

REF = reference_root()
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(REF is None, reason="reference package not installed "
                                 "(baseline/_ref or BOKT_REFERENCE_PATH)")]


@pytest.fixture(scope="module")
def overlay(tmp_path_factory):
    return dropin.overlay(REF, tmp_path_factory.mktemp("ref"))


def test_reference_gpu_correctness_tests(overlay, cuda_device):
    tests = overlay / "bo_kernel_tuner" / "tests" / "test_correctness.py"
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", str(tests), "-m", "gpu", "-q", "-p", "no:cacheprovider",
         "--rootdir", str(overlay)],
        env=dict(overlay_env(overlay), BO_TEST_CUDA_DEVICE=str(cuda_device.index)),
        capture_output=True, text=True, timeout=1800, cwd=str(overlay))
    tail = (proc.stdout + proc.stderr)[-3000:]
    assert proc.returncode == 0, tail
    assert " passed" in proc.stdout and "skipped" not in proc.stdout.split("\n")[-2], tail


@pytest.mark.parametrize("kernel,shape", [
    ("gemm", ["--m", "256", "--n", "512", "--k", "384"]),
    ("rmsnorm", ["--m", "512", "--n", "4096"]),
    ("moe_grouped_gemm", ["--n", "256", "--k", "128", "--expert-tokens", "0,1,33,0,9"]),
])
def test_reference_cli_tunes_these_kernels(kernel, shape, overlay, tmp_path, cuda_device):
    out = tmp_path / "study"
    proc = subprocess.run(
        [sys.executable, "-m", "bo_kernel_tuner.run_benchmark", "--kernel", kernel, "--mode",
         "tune", "--method", "grid", "--dtype", "bf16", *shape, "--seeds", "0", "--trials", "3",
         "--profile", "smoke", "--warmup", "2", "--repeats", "3", "--batch", "2",
         "--validation-seeds", "2", "--device", str(cuda_device.index), "--output", str(out)],
        env=overlay_env(overlay), capture_output=True, text=True, timeout=1800,
        cwd=str(tmp_path))
    assert proc.returncode == 0, (proc.stdout + proc.stderr)[-3000:]
    data = json.loads((out / "grid-seed-0" / "result.json").read_text())
    assert data["status"] == "complete" and data["attempts"] == 3
    assert data["successful_evaluations"] >= 1
    m = data["best"]["attrs"]["measurement"]
    assert m["latency_ms"] > 0 and len(m["validation"]) == 2
    assert m["compiled_shared_bytes"] > 0 and m["compiled_registers"] > 0
    assert m["compiled_spills"] == 0
    # Trial logs are the reference worker's (subprocess isolation per trial).
    assert len(list((out / "grid-seed-0" / "logs").glob("trial-*.log"))) == 3
