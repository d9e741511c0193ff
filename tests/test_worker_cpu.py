"""Host logic of the measurement worker (no GPU): input draw, FP32 gate, statistics."""

import math

import numpy as np
import pytest
import torch

from flashattentionanycard_b200.configs.search_spaces import Workload
from flashattentionanycard_b200.tuner import worker
from tests.golden_cases import kernel_cases, parse_key

CASES = kernel_cases()


@pytest.mark.parametrize("key", sorted(CASES))
def test_input_draw_matches_reference_fixture(key):
    """generate_inputs reproduces the reference's worker.prepare draw bit for bit
    (same generator, order and dtype), and reference_output its FP32 formula."""
    kernel, dtype, (m, n, k), seed = parse_key(key)
    case = CASES[key]
    tokens = (0, 1, 33, 0, 9)
    if kernel == "moe_grouped_gemm":
        starts = case["starts"].tolist()
        tokens = tuple(starts[i + 1] - starts[i] for i in range(len(starts) - 1))
    w = Workload(kernel, m, n, k, dtype, tokens)
    inputs = worker.generate_inputs(w, seed)
    for name, value in inputs.items():
        if name == "starts":
            assert value == case["starts"].tolist()
        else:
            assert np.array_equal(value.view(torch.int16).numpy().view(np.uint16), case[name])
    ref = worker.reference_output(w, inputs)
    assert torch.equal(ref, torch.from_numpy(case["ref"]))


def test_check_output_gate():
    ref = torch.randn(64, 64, generator=torch.Generator().manual_seed(1)) * 4
    out = ref.to(torch.bfloat16)
    stats = worker.check_output(out, ref, "bf16")
    assert stats["rtol"] == 0.02 and stats["atol"] == 0.15 and stats["normwise_rel_error"] < 4e-3
    bad = out.clone()
    bad[1, 1] = bad[1, 1] + 2.0
    with pytest.raises(AssertionError):
        worker.check_output(bad, ref, "bf16")
    nan = out.clone()
    nan[0, 0] = float("nan")
    with pytest.raises(AssertionError):
        worker.check_output(nan, ref, "bf16")
    assert worker.check_output(ref.half(), ref, "fp16")["atol"] == 0.02


def test_measurement_and_statistics_validation():
    with pytest.raises(ValueError):
        worker.Measurement(warmup=0)
    with pytest.raises(ValueError):
        worker.Measurement(repeats=2.0)
    s = worker.sample_statistics([1.0, 2.0, 4.0])
    assert s["latency_ms"] == 2.0 and s["mad_ms"] == 1.0
    for bad in ([1.0, 2.0], [1.0, 2.0, math.nan], [1.0, 2.0, -1.0]):
        with pytest.raises(ValueError):
            worker.sample_statistics(bad)


def test_implementation_labels():
    with pytest.raises(ValueError):
        worker.prepare(Workload("gemm", 8, 8, 8), torch.device("cpu"), 0, 1, "cutlass")
    # the torch baseline runs on CPU (as the reference's tests/test_confirmation.py:219-228)
    w = Workload("rmsnorm", 4, 16, 1, "bf16")
    call, out, ref = worker.prepare(w, torch.device("cpu"), 0, 1, "torch")
    assert out is None
    worker.check_output(call({}), ref, "bf16")


def test_worker_main_reports_errors(tmp_path):
    src, dst = tmp_path / "in.json", tmp_path / "out.json"
    src.write_text('{"workload": {"kernel": "nope"}}')
    import sys

    argv = sys.argv
    sys.argv = ["worker", str(src), str(dst)]
    try:
        worker.main()
    finally:
        sys.argv = argv
    import json

    result = json.loads(dst.read_text())
    assert result["status"] == "error" and result["error_type"] and "error" in result
