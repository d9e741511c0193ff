"""Parity at the benchmark configurations' full sizes.

Small configurations are checked element by element against the oracle.  The
8192^3 GEMM and the 64-expert MoE are checked on sampled rows and columns
(each sampled output row is a full dot-product row recomputed on the CPU), so
the comparison is exact in coverage of K and independent of problem size.
Tolerance: the reference gate (bf16 rtol 0.02 / atol 0.15, fp16 rtol 0.01 /
atol 0.02) and normwise relative error <= 1e-2.
"""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native, workloads
from flashattentionanycard_b200.configs.search_spaces import default_params
from flashattentionanycard_b200.kernels import gemm, moe_grouped_gemm, rmsnorm
from flashattentionanycard_b200.kernels.moe_routing import MoeRouter, gather_rows
from oracle import numerics, routing
from tests.gpu_helpers import as_f32, gate, nan_like

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def clean_status(cuda_device):
    _native.device_status(reset=True)
    yield
    assert _native.device_status(reset=True)[0] == 0


def test_gemm_smoke_127x193x257(cuda_device):
    a, b = workloads.gemm_inputs(127, 193, 257, "bf16", seed=0, scaled=False)
    out = nan_like((127, 193), "bf16", cuda_device)
    gemm.launch(a.to(cuda_device), b.to(cuda_device), out, default_params("gemm"))
    torch.cuda.synchronize()
    gate(out, numerics.gemm_fp32(as_f32(a), as_f32(b)), "bf16")


@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4])
def test_rmsnorm_4096(seed, cuda_device):
    x, w = workloads.rmsnorm_inputs(4096, 4096, "bf16", seed)
    out = nan_like((4096, 4096), "bf16", cuda_device)
    rmsnorm.launch(x.to(cuda_device), w.to(cuda_device), out, default_params("rmsnorm"), 1e-6)
    torch.cuda.synchronize()
    stats = gate(out, numerics.rmsnorm_fp32(as_f32(x), as_f32(w), 1e-6), "bf16")
    assert stats["normwise_rel_error"] < 5e-3


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_gemm_2048(dtype, cuda_device):
    a, b = workloads.gemm_inputs(2048, 2048, 2048, dtype, seed=0)
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    for p in (default_params("gemm"), dict(default_params("gemm"), BLOCK_N=128, num_stages=6)):
        out = nan_like((2048, 2048), dtype, cuda_device)
        gemm.launch(a.to(cuda_device), b.to(cuda_device), out, p)
        torch.cuda.synchronize()
        gate(out, ref, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_gemm_8192_sampled(dtype, cuda_device):
    n = 8192
    a, b = workloads.gemm_inputs(n, n, n, dtype, seed=0)
    out = nan_like((n, n), dtype, cuda_device)
    gemm.launch(a.to(cuda_device), b.to(cuda_device), out, default_params("gemm"))
    torch.cuda.synchronize()
    assert not torch.isnan(out).any().item()
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(n, 192, replace=False))
    cols = np.sort(rng.choice(n, 192, replace=False))
    af, bf = as_f32(a), as_f32(b)
    gate(out[torch.from_numpy(rows).to(cuda_device)], numerics.gemm_fp32(af[rows], bf), dtype)
    gate(out[:, torch.from_numpy(cols).to(cuda_device)], numerics.gemm_fp32(af, bf[:, cols]), dtype)


def test_moe_small(cuda_device):
    counts = workloads.MOE_SMALL_COUNTS
    cfg = workloads.MOE_SMALL
    x, w = workloads.moe_inputs(counts, cfg["k"], cfg["n"], "bf16", seed=0)
    starts = workloads.offsets_from_counts(counts)
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    offsets = torch.tensor(starts, dtype=torch.int32, device=cuda_device)
    for p in (default_params("moe_grouped_gemm"),
              dict(default_params("moe_grouped_gemm"), BLOCK_N=128, num_stages=5, CTA_MULTIPLIER=2)):
        out = nan_like((x.shape[0], cfg["n"]), "bf16", cuda_device)
        moe_grouped_gemm.launch(x.to(cuda_device), w.to(cuda_device), offsets, out, p, 148)
        torch.cuda.synchronize()
        gate(out, ref, "bf16")


def test_moe_large_routed_sampled(cuda_device):
    """64 experts, 16384 tokens top-2 Zipf(1.1): device routing bit-exact with
    the oracle; grouped GEMM on sampled rows of every non-empty expert."""
    x, w, ids = workloads.moe_large_inputs("bf16", seed=0, device=cuda_device)
    cfg = workloads.MOE_LARGE
    flat = ids.reshape(-1)
    a = flat.numel()
    r = MoeRouter(a, cfg["experts"], cuda_device)
    r(flat.to(cuda_device))
    packed = torch.empty(a, cfg["k"], device=cuda_device, dtype=torch.bfloat16)
    gather_rows(x, r.perm, packed, divisor=cfg["topk"])
    y = nan_like((a, cfg["n"]), "bf16", cuda_device)
    moe_grouped_gemm.launch(packed, w, r.offsets, y, default_params("moe_grouped_gemm"), 148)
    torch.cuda.synchronize()
    counts, offsets, perm, inv = routing.route(flat.numpy(), cfg["experts"])
    assert np.array_equal(r.counts.cpu().numpy(), counts)
    assert np.array_equal(r.perm.cpu().numpy(), perm)
    assert np.array_equal(r.inv_perm.cpu().numpy(), inv)
    assert not torch.isnan(y).any().item()
    rng = np.random.default_rng(1)
    for e in range(cfg["experts"]):
        s, t = int(offsets[e]), int(offsets[e + 1])
        if t == s:
            continue
        rows = np.unique(np.concatenate([[s, t - 1], rng.integers(s, t, size=6)]))
        tokens = perm[rows] // cfg["topk"]
        xs = as_f32(x[torch.from_numpy(tokens).to(cuda_device)])
        ref = numerics.gemm_fp32(xs, as_f32(w[e]))
        gate(y[torch.from_numpy(rows).to(cuda_device)], ref, "bf16")
