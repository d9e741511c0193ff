"""Pin the CPU oracle against the reference's own outputs (tests/golden) — CPU only."""

import numpy as np
import pytest

from oracle import numerics, routing
from tests.golden_cases import kernel_cases, parse_key, routing_cases

KERNEL_CASES = kernel_cases()
ROUTING_CASES = routing_cases()


def oracle_output(kernel, dtype, case):
    if kernel == "gemm":
        return numerics.gemm_fp32(numerics.to_f32(case["a"], dtype), numerics.to_f32(case["b"], dtype))
    if kernel == "rmsnorm":
        return numerics.rmsnorm_fp32(
            numerics.to_f32(case["x"], dtype), numerics.to_f32(case["weight"], dtype), 1e-6
        )
    return numerics.grouped_gemm_fp32(
        numerics.to_f32(case["x"], dtype), numerics.to_f32(case["weight"], dtype), case["starts"]
    )


@pytest.mark.parametrize("key", sorted(KERNEL_CASES))
def test_oracle_matches_reference_fp32(key):
    """The oracle restates worker.py:64,73-74,88-90: agree with the reference's
    own FP32 output to fp32 rounding (summation order may differ)."""
    kernel, dtype, _, _ = parse_key(key)
    case = KERNEL_CASES[key]
    mine = oracle_output(kernel, dtype, case)
    ref = case["ref"]
    assert mine.shape == ref.shape
    np.testing.assert_allclose(mine, ref, rtol=2e-5, atol=2e-5 * max(1.0, float(np.abs(ref).max())))


@pytest.mark.parametrize("key", sorted(k for k, v in KERNEL_CASES.items() if "triton" in v))
def test_reference_triton_kernel_passes_oracle_gate(key):
    """The reference's actual Triton kernel output (CPU interpreter) passes the
    gate against the oracle, and sits within one rounding step of it."""
    kernel, dtype, _, _ = parse_key(key)
    case = KERNEL_CASES[key]
    ref = oracle_output(kernel, dtype, case)
    out = numerics.to_f32(case["triton"], dtype)
    stats = numerics.check_output(out, ref, dtype)
    assert stats["normwise_rel_error"] < 1e-2
    rounded = numerics.round_to(ref, dtype)
    ulp = np.abs(rounded) * (2.0**-7 if dtype == "bf16" else 2.0**-10) + 1e-6
    assert np.all(np.abs(out - rounded) <= 2 * ulp + 1e-3 * np.abs(ref).max())


def test_gate_rejects_planted_error():
    """A wrong answer planted in the oracle's output fails the gate."""
    case = KERNEL_CASES["gemm|bf16|64x128x64|0"]
    ref = oracle_output("gemm", "bf16", case)
    bad = ref.copy()
    bad[3, 5] += 1.0
    with pytest.raises(AssertionError):
        numerics.check_output(bad, ref, "bf16")
    nan = ref.copy()
    nan[0, 0] = np.nan
    with pytest.raises(AssertionError):
        numerics.check_output(nan, ref, "bf16")


def test_bf16_conversion_matches_torch():
    torch = pytest.importorskip("torch")
    x = torch.randn(4096, generator=torch.Generator().manual_seed(0)) * 100
    x[:4] = torch.tensor([0.0, -0.0, 1e-40, 3.3895e38])
    ref_bits = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(numerics.f32_to_bf16_bits(x.numpy()), ref_bits)
    back = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(numerics.bf16_bits_to_f32(ref_bits), back)
    h_bits = x.to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(numerics.f32_to_fp16_bits(x.numpy()), h_bits)


@pytest.mark.parametrize("key", sorted(ROUTING_CASES))
def test_routing_oracle_matches_golden(key):
    case = ROUTING_CASES[key]
    experts = int(key.split("|")[2])
    counts, offsets, perm, inv = routing.route(case["ids"], experts)
    assert np.array_equal(counts, case["counts"])
    assert np.array_equal(offsets, case["offsets"])
    assert np.array_equal(perm, case["perm"])
    assert np.array_equal(inv[perm], np.arange(perm.size))


def test_routing_edge_cases():
    # all assignments on one expert, empty experts at both ends
    ids = np.full(37, 2, dtype=np.int32)
    counts, offsets, perm, inv = routing.route(ids, 5)
    assert counts.tolist() == [0, 0, 37, 0, 0]
    assert offsets.tolist() == [0, 0, 0, 37, 37, 37]
    assert perm.tolist() == list(range(37))
    # empty input
    counts, offsets, perm, inv = routing.route(np.zeros(0, dtype=np.int32), 3)
    assert counts.tolist() == [0, 0, 0] and offsets.tolist() == [0, 0, 0, 0] and perm.size == 0
    with pytest.raises(ValueError):
        routing.route(np.array([0, 3], dtype=np.int32), 3)


def test_grouped_oracle_leaves_uncovered_rows():
    x = np.ones((6, 2), np.float32)
    w = np.ones((2, 2, 3), np.float32)
    out = numerics.grouped_gemm_fp32(x, w, [1, 3, 5])
    assert np.isnan(out[0]).all() and np.isnan(out[5]).all()
    assert np.all(out[1:5] == 2.0)


def test_topk_gate_oracle_against_sorting():
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((50, 64)).astype(np.float32)
    logits[3, [5, 9]] = 7.0  # a tie: the lower index comes first
    ids, gates = routing.topk_gate(logits, 2)
    for t in range(50):
        want = sorted(range(64), key=lambda e: (-float(logits[t, e]), e))[:2]
        assert ids[t].tolist() == want
    assert ids[3].tolist() == [5, 9]
    np.testing.assert_allclose(gates.sum(axis=1), 1.0, rtol=1e-6)
    raw_ids, raw = routing.topk_gate(logits, 2, renormalize=False)
    assert np.array_equal(raw_ids, ids) and np.all(raw.sum(axis=1) < 1.0)


def test_combine_oracle():
    y = np.arange(12, dtype=np.float32).reshape(6, 2)
    gates = np.array([[0.5, 0.5], [1.0, 0.0], [0.25, 0.75]], np.float32)
    out = routing.combine(y, gates)
    assert np.allclose(out, [[1, 2], [4, 5], [0.25 * 8 + 0.75 * 10, 0.25 * 9 + 0.75 * 11]])
    perm_rows = np.array([5, 4, 3, 2, 1, 0])
    assert np.allclose(routing.combine(y, gates, perm_rows)[0], 0.5 * y[5] + 0.5 * y[4])


def test_fused_rmsnorm_gemm_restatement_is_exact_algebra():
    """The fused operator computes s[m] * (x[m] @ (w * b)) with s the per-row
    RMSNorm factor: in exact (float64) arithmetic this is the reference chain
    rmsnorm(x, w) @ b, so only the roundings differ."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((33, 40))
    w = 1 + 0.1 * rng.standard_normal(40)
    b = rng.standard_normal((40, 24)) / np.sqrt(40)
    eps = 1e-6
    chain = (x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + eps) * w) @ b
    s = 1 / np.sqrt(np.mean(x * x, axis=1) + eps)
    fused = s[:, None] * (x @ (w[:, None] * b))
    np.testing.assert_allclose(fused, chain, rtol=1e-12, atol=1e-12)
    ref32 = numerics.rmsnorm_gemm_fp32(x, w, b, eps)
    np.testing.assert_allclose(ref32, chain, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(numerics.rmsnorm_row_scale_fp32(x, eps), s, rtol=1e-6)


def test_timed_cpu_arm_matches_oracle():
    """The torch expressions the CPU arm times (oracle.reference_cpu) compute
    what the numpy oracle computes, on the 16-bit inputs of each kernel."""
    import torch

    from flashattentionanycard_b200 import workloads
    from oracle import reference_cpu

    threads = torch.get_num_threads()
    reference_cpu.configure(2)
    assert torch.get_num_threads() == 2
    torch.set_num_threads(threads)
    a, b = workloads.gemm_inputs(64, 96, 80, "bf16", seed=1)
    np.testing.assert_allclose(reference_cpu.gemm(a, b).numpy(),
                               numerics.gemm_fp32(a.float().numpy(), b.float().numpy()),
                               rtol=1e-5, atol=1e-5)
    x, w = workloads.rmsnorm_inputs(33, 200, "fp16", seed=2)
    np.testing.assert_allclose(reference_cpu.rmsnorm(x, w, 1e-6).numpy(),
                               numerics.rmsnorm_fp32(x.float().numpy(), w.float().numpy(), 1e-6),
                               rtol=1e-5, atol=1e-5)
    counts = (0, 5, 17, 0, 9)
    x, w = workloads.moe_inputs(counts, 48, 40, "bf16", seed=3)
    starts = workloads.offsets_from_counts(counts)
    np.testing.assert_allclose(reference_cpu.grouped_gemm(x, w, starts).numpy(),
                               numerics.grouped_gemm_fp32(x.float().numpy(), w.float().numpy(),
                                                          starts),
                               rtol=1e-5, atol=1e-5)
