"""The tcgen05 edge kernel: GEMM shapes whose row strides TMA cannot describe
(K % 8 or N % 8 != 0) and operands whose base is not 16-byte aligned, dense
and grouped, against the oracle.

Tolerance: the reference's FP32 gate, fp16 rtol 0.01 / atol 0.02 and bf16 rtol
0.02 / atol 0.15 (reference worker.py:111), plus a normwise relative error
<= 1e-2.  Outputs are NaN-prefilled so an unwritten element fails."""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native
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


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(127, 193, 257), (37, 77, 93), (1, 1, 1), (300, 130, 7),
                                   (129, 65, 1000), (1000, 3, 64), (5, 200, 2)])
def test_edge_shapes_on_tensor_cores(shape, dtype, cuda_device):
    m, n, k = shape
    g = torch.Generator().manual_seed(m + 3 * n + 7 * k)
    a = torch.randn(m, k, generator=g).to(TD[dtype])
    b = torch.randn(k, n, generator=g).to(TD[dtype])
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    out = nan_like((m, n), dtype, cuda_device)
    compiled = gemm.launch(a.to(cuda_device), b.to(cuda_device), out, {})
    torch.cuda.synchronize()
    assert compiled.path == "tcgen05_edge"
    gate(out, ref, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_misaligned_operands(dtype, cuda_device):
    """K and N multiples of 8 but every base pointer 2 bytes past a 16-byte
    boundary (views into larger buffers): the edge kernel, same results."""
    m, n, k = 200, 136, 264
    g = torch.Generator().manual_seed(1)
    a = torch.randn(m * k + 1, generator=g).to(TD[dtype]).to(cuda_device)[1:].view(m, k)
    b = torch.randn(k * n + 1, generator=g).to(TD[dtype]).to(cuda_device)[1:].view(k, n)
    outbuf = torch.full((m * n + 1,), float("nan"), dtype=TD[dtype], device=cuda_device)
    out = outbuf[1:].view(m, n)
    compiled = gemm.launch(a, b, out, {})
    torch.cuda.synchronize()
    assert compiled.path == "tcgen05_edge"
    gate(out, numerics.gemm_fp32(as_f32(a.cpu()), as_f32(b.cpu())), dtype)
    assert torch.isnan(outbuf[0]), "wrote outside the output"


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("counts", [(0, 1, 33, 0, 9), (0, 1, 17, 65), (130, 0, 0, 1, 257, 3)])
def test_grouped_edge(counts, dtype, cuda_device):
    k, n = 93, 77
    g = torch.Generator().manual_seed(sum(counts))
    t = sum(counts)
    x = torch.randn(t, k, generator=g).to(TD[dtype])
    w = torch.randn(len(counts), k, n, generator=g).to(TD[dtype])
    starts = np.concatenate([[0], np.cumsum(counts)]).tolist()
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    for off_dtype in (torch.int32, torch.int64):
        out = nan_like((t, n), dtype, cuda_device)
        offsets = torch.tensor(starts, dtype=off_dtype, device=cuda_device)
        moe_grouped_gemm.launch(x.to(cuda_device), w.to(cuda_device), offsets, out, {}, 148)
        torch.cuda.synchronize()
        gate(out, ref, dtype)


def test_grouped_edge_leaves_rows_outside_experts(cuda_device):
    """Offsets covering rows [2, 40) of 50: rows outside stay untouched."""
    k, n = 20, 30
    x = torch.randn(50, k).bfloat16().to(cuda_device)
    w = torch.randn(2, k, n).bfloat16().to(cuda_device)
    offsets = torch.tensor([2, 20, 40], dtype=torch.int32, device=cuda_device)
    out = torch.full((50, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    moe_grouped_gemm.launch(x, w, offsets, out, {}, 148)
    torch.cuda.synchronize()
    assert torch.isnan(out[:2]).all() and torch.isnan(out[40:]).all()
    ref = numerics.grouped_gemm_fp32(as_f32(x[2:40].cpu()), as_f32(w.cpu()), [0, 18, 38])
    gate(out[2:40], ref, "bf16")
