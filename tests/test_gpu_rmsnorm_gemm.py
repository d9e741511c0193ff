"""Fused RMSNorm -> GEMM against the oracle on a B200.

Oracle: the reference's FP32 formulas composed, rmsnorm (worker.py:73-74) then
the matmul (worker.py:64), in fp32 on the CPU (oracle.numerics.rmsnorm_gemm_fp32).
Gate: the reference's tolerance for the output dtype (bf16 rtol 0.02 / atol 0.15,
fp16 rtol 0.01 / atol 0.02) plus normwise relative error <= 1e-2.
"""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import workloads
from flashattentionanycard_b200.kernels import gemm, rmsnorm, rmsnorm_gemm
from oracle import numerics
from tests.gpu_helpers import as_f32, gate, nan_like

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "fp16": torch.float16}

PARAMS = [
    {"BLOCK_N": 256, "num_stages": 6, "GROUP_M": 8, "CTA_GROUP": 2},
    {"BLOCK_N": 128, "num_stages": 8, "GROUP_M": 4, "CTA_GROUP": 2},
    {"BLOCK_N": 256, "num_stages": 4, "GROUP_M": 8, "CTA_GROUP": 1},
    {"BLOCK_N": 128, "num_stages": 3, "GROUP_M": 1, "CTA_GROUP": 1},
    {"BLOCK_N": 64, "num_stages": 2, "GROUP_M": 16, "CTA_GROUP": 1},
]


def oracle(x, w, b, eps):
    return numerics.rmsnorm_gemm_fp32(as_f32(x), as_f32(w), as_f32(b), eps)


def to_dev(dev, *ts):
    return [t.to(dev) for t in ts]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 8, 8), (128, 64, 256), (300, 1000, 520), (257, 4104, 136),
                                   (1024, 2048, 1024)])
def test_fused_matches_oracle(shape, dtype, cuda_device):
    m, k, n = shape
    x, w, b = workloads.rmsnorm_gemm_inputs(m, k, n, dtype, seed=m + k)
    ref = oracle(x, w, b, 1e-6)
    xd, wd, bd = to_dev(cuda_device, x, w, b)
    folded = rmsnorm_gemm.fold_weight(wd, bd)
    for p in PARAMS:
        out = nan_like((m, n), dtype, cuda_device)
        compiled = rmsnorm_gemm.launch(xd, folded, out, p, 1e-6)
        torch.cuda.synchronize()
        assert compiled.path == "tcgen05" and compiled.n_spills == 0
        gate(out, ref, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_fold_is_the_rounded_product(dtype, cuda_device):
    """b_folded[k, n] is weight[k] * b[k, n] rounded once to the dtype: bit-exact
    against torch's fp32 product rounded to the same dtype."""
    x, w, b = workloads.rmsnorm_gemm_inputs(8, 264, 1032, dtype, seed=5)
    wd, bd = to_dev(cuda_device, w, b)
    folded = rmsnorm_gemm.fold_weight(wd, bd)
    want = (wd.float().unsqueeze(1) * bd.float()).to(DT[dtype])
    torch.cuda.synchronize()
    assert torch.equal(folded, want)


@pytest.mark.parametrize("eps", [0.0, 1e-6, 1e-2])
def test_row_scale_against_oracle(eps, cuda_device):
    m, k = 777, 4096
    x, _, _ = workloads.rmsnorm_gemm_inputs(m, k, 8, "bf16", seed=2)
    x = (x.float() * torch.logspace(-3, 3, m).unsqueeze(1)).bfloat16()
    s = torch.empty(m, device=cuda_device, dtype=torch.float32)
    rmsnorm_gemm.row_scale(x.to(cuda_device), s, eps)
    want = numerics.rmsnorm_row_scale_fp32(as_f32(x), eps)
    np.testing.assert_allclose(s.cpu().numpy(), want, rtol=2e-6)


@pytest.mark.parametrize("eps", [0.0, 1e-6, 1e-2, 0.5])
def test_epsilon_and_row_magnitudes(eps, cuda_device):
    """Rows of very different magnitude (and an all-zero row when eps > 0,
    whose output is exactly zero) all match the oracle."""
    m, k, n = 256, 512, 256
    x, w, b = workloads.rmsnorm_gemm_inputs(m, k, n, "bf16", seed=3)
    x = (x.float() * torch.logspace(-3, 3, m).unsqueeze(1)).bfloat16()
    if eps > 0:
        x[7] = 0
    ref = oracle(x, w, b, eps)
    xd, wd, bd = to_dev(cuda_device, x, w, b)
    out = nan_like((m, n), "bf16", cuda_device)
    rmsnorm_gemm.launch(xd, rmsnorm_gemm.fold_weight(wd, bd), out, PARAMS[0], eps)
    torch.cuda.synchronize()
    gate(out, ref, "bf16")
    if eps > 0:
        assert torch.count_nonzero(out[7]).item() == 0


def test_fused_and_unfused_chain_agree(cuda_device):
    """The fused operator and the two-call chain it replaces (our rmsnorm,
    then our GEMM) both pass the gate and agree to bf16 rounding."""
    m, k, n = 1024, 4096, 2048
    x, w, b = workloads.rmsnorm_gemm_inputs(m, k, n, "bf16", seed=11)
    ref = oracle(x, w, b, 1e-6)
    xd, wd, bd = to_dev(cuda_device, x, w, b)
    fused = nan_like((m, n), "bf16", cuda_device)
    rmsnorm_gemm.launch(xd, rmsnorm_gemm.fold_weight(wd, bd), fused, PARAMS[0], 1e-6)
    xn = torch.empty_like(xd)
    rmsnorm.launch(xd, wd, xn, {"ROWS_PER_CTA": 1, "num_warps": 4, "num_stages": 1}, 1e-6)
    chain = nan_like((m, n), "bf16", cuda_device)
    gemm.launch(xn, bd, chain, PARAMS[0])
    torch.cuda.synchronize()
    gate(fused, ref, "bf16")
    gate(chain, ref, "bf16")
    assert (fused.float() - chain.float()).abs().max().item() <= 0.05 * float(np.abs(ref).max())


def test_full_size_workload_properties(cuda_device):
    """The bench shape (x [4096, 4096] -> [4096, 14336]): sampled rows against
    the oracle; rows of x scaled by 4 keep their outputs at the oracle's (RMSNorm
    is scale invariant up to eps) and every other row is bit-identical (rows are
    independent in the row-scale pass and inside a GEMM tile)."""
    cfg = workloads.RMSNORM_GEMM
    m, k, n = cfg["m"], cfg["k"], cfg["n"]
    x, w, b = workloads.rmsnorm_gemm_inputs(m, k, n, "bf16", seed=0)
    xd, wd, bd = to_dev(cuda_device, x, w, b)
    folded = rmsnorm_gemm.fold_weight(wd, bd)
    out = nan_like((m, n), "bf16", cuda_device)
    rmsnorm_gemm.launch(xd, folded, out, PARAMS[0], cfg["eps"])
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    rows = np.random.default_rng(0).choice(m, 48, replace=False)
    ref = oracle(x[rows], w, b, cfg["eps"])
    gate(out[rows], ref, "bf16")
    x2 = xd.clone()
    x2[rows] = (x2[rows].float() * 4.0).bfloat16()  # exact in bf16
    out2 = nan_like((m, n), "bf16", cuda_device)
    rmsnorm_gemm.launch(x2, folded, out2, PARAMS[0], cfg["eps"])
    torch.cuda.synchronize()
    gate(out2[rows], ref, "bf16")
    keep = torch.ones(m, dtype=torch.bool, device=cuda_device)
    keep[torch.as_tensor(rows, device=cuda_device)] = False
    assert torch.equal(out2[keep], out[keep])


def test_graph_capture_after_first_call(cuda_device):
    m, k, n = 512, 1024, 512
    x, w, b = workloads.rmsnorm_gemm_inputs(m, k, n, "bf16", seed=9)
    xd, wd, bd = to_dev(cuda_device, x, w, b)
    folded = rmsnorm_gemm.fold_weight(wd, bd)
    out = nan_like((m, n), "bf16", cuda_device)
    rmsnorm_gemm.launch(xd, folded, out, PARAMS[0])
    torch.cuda.synchronize()
    first = out.clone()
    out.fill_(float("nan"))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=s):
        rmsnorm_gemm.launch(xd, folded, out, PARAMS[0])
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)


def test_back_to_back_launches_use_their_own_row_scales(cuda_device):
    """The row-scaled GEMM's main loop may overlap the row-scale pass in front
    of it; its epilogue must still see that pass's scales.  Alternate x and 4x
    (exact in bf16, same normalised rows) through one workspace in a graph of
    back-to-back launches: a stale scale would show as a 4x or 1/4x output."""
    m, k, n = 2048, 4096, 2048
    x, w, b = workloads.rmsnorm_gemm_inputs(m, k, n, "bf16", seed=21)
    xd, wd, bd = to_dev(cuda_device, x, w, b)
    x4 = (xd.float() * 4).bfloat16()
    folded = rmsnorm_gemm.fold_weight(wd, bd)
    ws = torch.empty(m, device=cuda_device, dtype=torch.float32)
    outs = [torch.empty(m, n, device=cuda_device, dtype=torch.bfloat16) for _ in range(12)]
    rmsnorm_gemm.launch(xd, folded, outs[0], PARAMS[0], 1e-6, scale_workspace=ws)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.graph(g, stream=s):
        for i, o in enumerate(outs):
            rmsnorm_gemm.launch(x4 if i % 2 else xd, folded, o, PARAMS[0], 1e-6,
                                scale_workspace=ws)
    g.replay()
    torch.cuda.synchronize()
    ref = outs[0].float()
    for o in outs[1:]:
        assert (o.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item()


def test_unsupported_shapes_raise(cuda_device):
    x = torch.randn(16, 12, device=cuda_device).bfloat16()  # K % 8 != 0
    w = torch.ones(12, device=cuda_device).bfloat16()
    b = torch.randn(12, 16, device=cuda_device).bfloat16()
    out = torch.empty(16, 16, device=cuda_device).bfloat16()
    folded = rmsnorm_gemm.fold_weight(w, b)
    with pytest.raises(RuntimeError, match="multiples of 8"):
        rmsnorm_gemm.launch(x, folded, out, PARAMS[0])
    with pytest.raises(ValueError):
        rmsnorm_gemm.fold_weight(w[:8], b)
