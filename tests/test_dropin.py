"""The reference's own modules bound to these kernels by the five-file overlay
(flashattentionanycard_b200.dropin), checked without a GPU."""

import json
import subprocess
import sys

import pytest

from flashattentionanycard_b200 import dropin
from tests.dropin import overlay_env, reference_root

REF = reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="reference package not installed "
                                "(baseline/_ref or BOKT_REFERENCE_PATH)")


@pytest.fixture
def overlay(tmp_path):
    return dropin.overlay(REF, tmp_path / "ref")


def run(code, overlay, *args):
    return subprocess.run([sys.executable, *args] if not code else [sys.executable, "-c", code],
                          env=overlay_env(overlay), capture_output=True, text=True, timeout=300)


def test_overlay_binds_these_kernels(overlay):
    code = """
import json
import bo_kernel_tuner.kernels.gemm as g, bo_kernel_tuner.kernels.rmsnorm as r
import bo_kernel_tuner.kernels.moe_grouped_gemm as m
from bo_kernel_tuner.configs.search_spaces import Workload, search_space
from bo_kernel_tuner.tuner.hardware import Hardware, prune_reason
from bo_kernel_tuner.tuner import worker
print(json.dumps({"mods": [g.launch.__module__, r.launch.__module__, m.launch.__module__],
                  "workload": Workload.__module__, "hardware": Hardware.__module__,
                  "worker": worker.__file__, "space": sorted(search_space("gemm"))}))
"""
    proc = run(code, overlay)
    assert proc.returncode == 0, proc.stderr
    info = json.loads(proc.stdout.strip().splitlines()[-1])
    assert info["mods"] == ["flashattentionanycard_b200.kernels.gemm",
                            "flashattentionanycard_b200.kernels.rmsnorm",
                            "flashattentionanycard_b200.kernels.moe_grouped_gemm"]
    assert info["workload"] == "flashattentionanycard_b200.configs.search_spaces"
    assert info["hardware"] == "flashattentionanycard_b200.tuner.hardware"
    assert info["worker"].startswith(str(overlay))  # the reference's own worker
    assert "SPLIT_K" in info["space"] and "CTA_GROUP" in info["space"]


def test_overlay_leaves_the_rest_of_the_reference_alone(overlay):
    src = dropin.reference_package(REF)
    dst = overlay / "bo_kernel_tuner"
    for path in src.rglob("*.py"):
        rel = path.relative_to(src).as_posix()
        if rel in dropin.SHIMS:
            continue
        assert (dst / rel).read_bytes() == path.read_bytes(), rel


def test_reference_cli_dry_run_sees_the_cuda_space(overlay, tmp_path):
    proc = run(None, overlay, "-m", "bo_kernel_tuner.run_benchmark", "--dry-run", "--kernel",
               "gemm", "--mode", "tune", "--method", "grid", "--output", str(tmp_path / "o"))
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "grid_size" in proc.stdout and not (tmp_path / "o").exists()


def test_overlay_refuses_existing_destination(overlay):
    with pytest.raises(FileExistsError):
        dropin.overlay(REF, overlay)
