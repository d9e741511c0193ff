"""Contiguous FP16/BF16 GEMM on sm_100a tcgen05, FP32 accumulation, masked edge tiles.

Drop-in for the reference's ``bo_kernel_tuner/kernels/gemm.py:43-48``: same
``launch(a, b, out, params)`` signature and meaning (C[M,N] = A[M,K] @ B[K,N],
row-major contiguous, result rounded to ``out``'s dtype, every element of
``out`` written).  The tile order follows the reference's GROUP_M raster
(``gemm.py:20-26``) inside a persistent warp-specialised kernel.  With
``SPLIT_K`` > 1 the K loop of every tile is split across workers (split-K /
stream-K); the fp32 partials go through a per-device workspace allocated on
the first such call (``_native.splitk_workspace``), so that first call must
come before any graph capture.  From ``SPLIT_K`` 4 up the partials are summed
by a second kernel launched right after the GEMM on the same stream.
"""

import ctypes

from flashattentionanycard_b200 import _native


def launch(a, b, out, params):
    m, k = a.shape
    n = b.shape[1]
    if b.shape[0] != k or tuple(out.shape) != (m, n):
        raise ValueError(f"shape mismatch: a {tuple(a.shape)}, b {tuple(b.shape)}, out {tuple(out.shape)}")
    if not (a.dtype == b.dtype == out.dtype):
        raise ValueError("a, b and out must share one dtype")
    if not (a.is_contiguous() and b.is_contiguous() and out.is_contiguous()):
        raise ValueError("a, b and out must be contiguous row-major tensors")
    if not (a.is_cuda and b.is_cuda and out.is_cuda):
        raise ValueError("a, b and out must be CUDA tensors")
    lib = _native.load()
    dtype = _native.dtype_code(a.dtype)
    p = _native.make_params(params)
    ws, ws_bytes = _native.splitk_workspace(_native.KERNEL_GEMM, params, a.device)
    _native.check(
        lib.bokt_gemm_ex(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, dtype,
                         ctypes.byref(p), ws, ws_bytes, _native.current_stream(a.device)),
        "bokt_gemm",
    )
    # The library takes the edge kernel for any operand not 16-byte aligned;
    # report that kernel's attributes then (k = 1 selects it in the query).
    aligned = all(t.data_ptr() % 16 == 0 for t in (a, b, out))
    return _native.kernel_attrs(_native.KERNEL_GEMM, dtype, n, k if aligned else 1, params,
                                a.device.index)
