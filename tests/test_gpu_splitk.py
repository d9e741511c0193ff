"""Split-K / stream-K (SPLIT_K > 1) of the tcgen05 GEMM and grouped GEMM against the oracle.

Tolerance (every numeric test): the reference's FP32 gate, fp16 rtol 0.01 /
atol 0.02 and bf16 rtol 0.02 / atol 0.15 (reference worker.py:111), plus a
normwise relative error ||out - ref|| / ||ref|| <= 1e-2.  Outputs are
NaN-prefilled so an unwritten element fails.  A split run adds the same fp32
partials in the same order every time, so repeated runs are bit-identical.
"""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native, workloads
from flashattentionanycard_b200.kernels import gemm, moe_grouped_gemm
from oracle import numerics
from tests.gpu_helpers import as_f32, gate, nan_like

pytestmark = pytest.mark.gpu

TD = {"bf16": torch.bfloat16, "fp16": torch.float16}


@pytest.fixture(autouse=True)
def clean_status(cuda_device):
    _native.device_status(reset=True)
    yield
    code, detail = _native.device_status(reset=True)
    assert code == 0, f"device status {code} (detail {detail})"


def _inputs(m, n, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) / k ** 0.5).to(TD[dtype])
    b = torch.randn(k, n, generator=g).to(TD[dtype])
    return a, b


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("cta_group", [1, 2])
@pytest.mark.parametrize("split", [2, 3, 4, 8, 16, 32])
def test_dense_split_2048(split, cta_group, dtype, cuda_device):
    """2048^3 (64 pair tiles / 128 single tiles of 32 k-blocks on 74 pairs /
    148 CTAs: the partial-wave shape split-K is for), every split value."""
    a, b = workloads.gemm_inputs(2048, 2048, 2048, dtype, seed=0)
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    a, b = a.to(cuda_device), b.to(cuda_device)
    p = {"BLOCK_N": 256, "num_stages": 6 if cta_group == 2 else 4, "CTA_GROUP": cta_group,
         "SPLIT_K": split}
    outs = []
    for _ in range(2):
        out = nan_like((2048, 2048), dtype, cuda_device)
        gemm.launch(a, b, out, p)
        torch.cuda.synchronize()
        outs.append(out)
    gate(outs[0], ref, dtype)
    assert torch.equal(outs[0], outs[1]), "split-K result differs between identical runs"


SHAPES = [(1, 8, 64), (129, 136, 72), (300, 520, 1000), (257, 264, 4104), (1000, 64, 128),
          (640, 768, 2048), (4096, 512, 512)]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", SHAPES)
def test_dense_split_ragged(shape, dtype, cuda_device):
    """Ragged M/N/K tails, K of 1 to 65 k-blocks (split clamped to the k-block
    count), block_n 64/128/256, single CTAs and pairs."""
    m, n, k = shape
    a, b = _inputs(m, n, k, dtype, m * 7 + n)
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    a, b = a.to(cuda_device), b.to(cuda_device)
    for cta_group, bn in ((1, 64), (1, 128), (1, 256), (2, 128), (2, 256)):
        for split in (2, 4, 16):
            p = {"BLOCK_N": bn, "CTA_GROUP": cta_group, "SPLIT_K": split}
            out = nan_like((m, n), dtype, cuda_device)
            gemm.launch(a, b, out, p)
            torch.cuda.synchronize()
            gate(out, ref, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(256, 256, 65536), (128, 512, 32768), (300, 136, 20000)])
def test_dense_split_tall_k(shape, dtype, cuda_device):
    """Tall-K shapes (one to a few output tiles, hundreds of k-blocks) with
    the separate reduction, up to 128 slices: single CTAs and pairs, every
    split tile summed from up to 148 partials; repeated runs bit-identical."""
    m, n, k = shape
    a, b = _inputs(m, n, k, dtype, m + n)
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    a, b = a.to(cuda_device), b.to(cuda_device)
    for cta_group in (1, 2):
        for split in (4, 16, 64, 128):
            p = {"BLOCK_N": 128 if n % 256 else 256, "CTA_GROUP": cta_group, "SPLIT_K": split}
            outs = []
            for _ in range(2):
                out = nan_like((m, n), dtype, cuda_device)
                gemm.launch(a, b, out, p)
                torch.cuda.synchronize()
                outs.append(out)
            gate(outs[0], ref, dtype)
            assert torch.equal(outs[0], outs[1]), f"split {split} differs between identical runs"


def test_owner_fixup_and_separate_reduction_agree(cuda_device):
    """S = 3 (owner fix-up) and S = 4 (separate reduction) of one problem both
    pass the gate and agree to within a rounding step almost everywhere."""
    a, b = _inputs(512, 768, 8192, "bf16", 5)
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    a, b = a.to(cuda_device), b.to(cuda_device)
    outs = []
    for split in (3, 4):
        out = nan_like((512, 768), "bf16", cuda_device)
        gemm.launch(a, b, out, {"CTA_GROUP": 2, "SPLIT_K": split})
        torch.cuda.synchronize()
        gate(out, ref, "bf16")
        outs.append(out.float())
    diff = (outs[0] - outs[1]).abs()
    assert float((diff > outs[0].abs() * 2.0 ** -7 + 1e-6).float().mean()) < 1e-3


def test_split_graph_replay_and_shared_workspace(cuda_device):
    """Back-to-back split launches of four shapes (owner fix-up and separate
    reduction) share one workspace inside a CUDA graph replayed many times
    (the launch sequence number, not a cleared flag, tells a fresh partial
    from a stale one; a reduction finishes before the next GEMM writes)."""
    shapes = [(2048, 2048, 2048, 8), (512, 1024, 3072, 16), (1024, 1024, 2048, 2),
              (256, 256, 32768, 64)]
    data = []
    for m, n, k, s in shapes:
        a, b = _inputs(m, n, k, "bf16", m + k)
        ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
        data.append((a.to(cuda_device), b.to(cuda_device), ref, s,
                     torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)))
    params = [{"CTA_GROUP": 2, "SPLIT_K": s} for *_, s, _ in data]

    def step():
        for (a, b, _, _, out), p in zip(data, params):
            gemm.launch(a, b, out, p)

    step()  # allocates the workspace, sets kernel attributes
    torch.cuda.synchronize()
    first = [out.clone() for *_, out in data]
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(5):
            step()
    for _ in range(10):
        graph.replay()
    torch.cuda.synchronize()
    for (a, b, ref, _, out), f in zip(data, first):
        gate(out, ref, "bf16")
        assert torch.equal(out, f)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("counts", [(0, 16, 64, 256, 1024, 32, 8, 128), (0, 1, 33, 0, 9),
                                    (128, 0, 129, 1, 255), (0, 0, 0, 300)])
@pytest.mark.parametrize("split", [2, 4, 16])
def test_grouped_split(counts, split, dtype, cuda_device):
    """Single-CTA grouped GEMM with split-K over ragged and empty experts (the
    MoE small configuration first), int32 and int64 offsets."""
    k, n = (1024, 2048) if len(counts) == 8 else (256, 384)
    x, w = workloads.moe_inputs(counts, k, n, dtype, seed=3)
    starts = workloads.offsets_from_counts(counts)
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    for off_dtype in (torch.int32, torch.int64):
        offsets = torch.tensor(starts, dtype=off_dtype, device=cuda_device)
        p = {"BLOCK_N": 256, "num_stages": 4, "CTA_GROUP": 1, "SPLIT_K": split}
        out = nan_like((x.shape[0], n), dtype, cuda_device)
        moe_grouped_gemm.launch(xd, wd, offsets, out, p, 148)
        torch.cuda.synchronize()
        gate(out, ref, dtype)


def test_grouped_pairs_reject_split(cuda_device):
    x, w = workloads.moe_inputs((64, 64), 128, 256, "bf16", seed=0)
    offsets = torch.tensor([0, 64, 128], dtype=torch.int32, device=cuda_device)
    out = torch.empty(128, 256, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(RuntimeError, match="split_k"):
        moe_grouped_gemm.launch(x.to(cuda_device), w.to(cuda_device), offsets, out,
                                {"CTA_GROUP": 2, "SPLIT_K": 4}, 148)


def test_split_matches_unsplit_closely(cuda_device):
    """Split and unsplit results of one problem differ only by fp32 summation
    order: within one bf16 rounding step of each other almost everywhere."""
    a, b = _inputs(1024, 1024, 4096, "bf16", 11)
    a, b = a.to(cuda_device), b.to(cuda_device)
    outs = []
    for split in (1, 8):
        out = torch.empty(1024, 1024, dtype=torch.bfloat16, device=cuda_device)
        gemm.launch(a, b, out, {"CTA_GROUP": 2, "SPLIT_K": split})
        outs.append(out.float())
    torch.cuda.synchronize()
    diff = (outs[0] - outs[1]).abs()
    ulp = outs[0].abs() * 2.0 ** -7 + 1e-6
    assert float((diff > ulp).float().mean()) < 1e-3
    assert np.isfinite(float(diff.max()))
