"""The tuner plumbing end to end on the GPU: fresh worker process per trial
(subprocess isolation), grid search over launch parameters, and the engine's
command line."""

import json

import pytest

from flashattentionanycard_b200.configs.search_spaces import Workload
from flashattentionanycard_b200.tuner import engine
from flashattentionanycard_b200.tuner.hardware import Hardware
from flashattentionanycard_b200.tuner.worker import CANDIDATE, Measurement

pytestmark = pytest.mark.gpu


def test_isolated_worker_process(tmp_path, cuda_device):
    hw = Hardware.detect(cuda_device.index)
    result = engine.isolated_evaluate(
        Workload("gemm", 256, 512, 384, "bf16"), hw,
        {"BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_K": 64, "num_warps": 6, "num_stages": 3,
         "GROUP_M": 4, "CTA_GROUP": 2},
        Measurement(3, 3, 4, 2), 600, tmp_path, 0)
    assert result["status"] == "ok" and result["implementation"] == CANDIDATE
    assert result["latency_ms"] > 0 and len(result["validation"]) == 2
    assert result["compiled_path"] == "tcgen05" and result["compiled_spills"] == 0


def test_grid_search_in_worker_processes(tmp_path, cuda_device):
    hw = Hardware.detect(cuda_device.index)
    space = {"ROWS_PER_CTA": [1], "num_warps": [4, 8], "num_stages": [1]}
    result = engine.run_search(Workload("rmsnorm", 1024, 4096, 1, "bf16"), hw, space, "grid", 0,
                               4, tmp_path, Measurement(3, 3, 8, 1), trial_timeout=600)
    assert result["status"] == "complete" and result["attempts"] == 2
    assert result["successful_evaluations"] == 2
    assert json.loads((tmp_path / "result.json").read_text())["best"] == result["best"]


def test_cli_tune_run(tmp_path, cuda_device):
    out = tmp_path / "study"
    rc = engine.main([
        "--kernel", "moe_grouped_gemm", "--method", "grid", "--dtype", "bf16",
        "--n", "256", "--k", "128", "--expert-tokens", "0,1,33,0,9", "--trials", "2",
        "--profile", "smoke", "--measurement", "2,3,2,1", "--output", str(out),
        "--device", str(cuda_device.index)])
    assert rc == 0
    data = json.loads((out / "result.json").read_text())
    assert data["status"] == "complete" and data["attempts"] == 2
