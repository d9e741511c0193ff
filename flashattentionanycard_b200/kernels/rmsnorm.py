"""Fused RMS reduction, normalization, and weight multiplication on sm_100a.

Drop-in for the reference's ``bo_kernel_tuner/kernels/rmsnorm.py:29-33``:
``launch(x, weight, out, params, epsilon=1e-6)`` computes
``out = x * rsqrt(mean(x^2, -1) + epsilon) * weight`` in fp32 and stores in
``out``'s dtype; ``params`` holds ``ROWS_PER_CTA`` and ``num_warps`` as in the
reference's search space.
"""

import ctypes

from flashattentionanycard_b200 import _native


def launch(x, weight, out, params, epsilon=1e-6):
    m, n = x.shape
    if tuple(weight.shape) != (n,) or tuple(out.shape) != (m, n):
        raise ValueError(
            f"shape mismatch: x {tuple(x.shape)}, weight {tuple(weight.shape)}, out {tuple(out.shape)}"
        )
    if not (x.dtype == weight.dtype == out.dtype):
        raise ValueError("x, weight and out must share one dtype")
    if not (x.is_contiguous() and weight.is_contiguous() and out.is_contiguous()):
        raise ValueError("x, weight and out must be contiguous")
    if not (x.is_cuda and weight.is_cuda and out.is_cuda):
        raise ValueError("x, weight and out must be CUDA tensors")
    lib = _native.load()
    dtype = _native.dtype_code(x.dtype)
    p = _native.make_params(params)
    _native.check(
        lib.bokt_rmsnorm(x.data_ptr(), weight.data_ptr(), out.data_ptr(), m, n, float(epsilon),
                         dtype, ctypes.byref(p), _native.current_stream(x.device)),
        "bokt_rmsnorm",
    )
    return _native.kernel_attrs(_native.KERNEL_RMSNORM, dtype, n, 0, params, x.device.index)
