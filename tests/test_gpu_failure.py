"""Failure detection on the GPU without a GPU fault: a kernel waits on an
mbarrier nothing will complete; the bounded wait gives up after 50 ms, the
status word reports it, and the context keeps working."""

import ctypes

import pytest
import torch

from flashattentionanycard_b200 import _native
from flashattentionanycard_b200.kernels import gemm
from oracle import numerics
from tests.gpu_helpers import as_f32, gate

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives(cuda_device):
    lib = _native.load()
    _native.device_status(reset=True)
    gave_up = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    _native.check(lib.bokt_selftest_bounded_wait(50_000_000, gave_up.data_ptr(), stream),
                  "bokt_selftest_bounded_wait")
    torch.cuda.synchronize()
    assert gave_up.item() == 1
    assert _native.device_status(reset=True) == (1, 99)
    # The context is still usable: a tcgen05 GEMM right after is correct.
    a = torch.randn(256, 256).bfloat16()
    b = torch.randn(256, 256).bfloat16()
    out = torch.empty(256, 256, dtype=torch.bfloat16, device=cuda_device)
    gemm.launch(a.to(cuda_device), b.to(cuda_device), out, {"CTA_GROUP": 2})
    torch.cuda.synchronize()
    gate(out, numerics.gemm_fp32(as_f32(a), as_f32(b)), "bf16")
    assert _native.device_status(reset=True) == (0, 0)
    assert lib.bokt_selftest_bounded_wait(0, gave_up.data_ptr(), stream) == 1
