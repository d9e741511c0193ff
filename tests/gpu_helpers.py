"""Shared helpers of the GPU parity tests."""

import numpy as np
import torch

from oracle import numerics

TORCH_DTYPE = {"bf16": torch.bfloat16, "fp16": torch.float16}


def from_bits(bits, dtype, device):
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TORCH_DTYPE[dtype])
    return t.to(device)


def to_numpy_f32(t):
    return t.detach().float().cpu().numpy()


def as_f32(t):
    """Exact fp32 values of a CPU 16-bit tensor, as numpy."""
    return t.detach().float().cpu().numpy()


def nan_like(shape, dtype, device):
    return torch.full(shape, float("nan"), dtype=TORCH_DTYPE[dtype], device=device)


def gate(out, ref, dtype):
    """The reference's FP32 gate (fp16 rtol 0.01 / atol 0.02, bf16 rtol 0.02 /
    atol 0.15) and the normwise relative error bound 1e-2."""
    return numerics.check_output(to_numpy_f32(out), ref, dtype)
