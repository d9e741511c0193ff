"""RMSNorm fused with the GEMM that consumes it (sm_100a tcgen05).

Replaces the pair of reference operator calls

    rmsnorm.launch(x, weight, xn, params_norm, epsilon)   # kernels/rmsnorm.py:29-33
    gemm.launch(xn, b, out, params_gemm)                   # kernels/gemm.py:43-48

without writing ``xn`` to HBM.  The RMSNorm formula of ``kernels/rmsnorm.py:22-25``,
``xn = x * rsqrt(mean(x^2) + eps) * w``, is split into its per-column weight and
its per-row factor:

* ``fold_weight(weight, b)`` folds the weight into the GEMM's B once per weight
  pair: ``b_folded[k, n] = weight[k] * b[k, n]`` (rounded to the dtype);
* ``launch(x, b_folded, out, params, epsilon)`` runs one HBM-bound pass over x
  for ``s[m] = rsqrt(mean(x[m]^2) + epsilon)`` and the tcgen05 GEMM
  ``x @ b_folded`` whose epilogue scales accumulator row m by ``s[m]`` in fp32
  before rounding.

The GEMM's operand path is the plain GEMM's (TMA -> shared memory -> tcgen05),
so it runs at the plain GEMM's speed; the normalised activations are never
materialised.  ``params`` are the GEMM's (BLOCK_N, num_stages, GROUP_M,
CTA_GROUP, ...).  Shapes: x [M, K], weight [K], b / b_folded [K, N], out [M, N],
one dtype (fp16/bf16), K and N multiples of 8.
"""

import ctypes
import math
import threading

from flashattentionanycard_b200 import _native

_lock = threading.Lock()
_row_scale = {}  # (device index, M) -> fp32 workspace, created on first use


def _check(tensors, names):
    if len({t.dtype for t in tensors}) != 1:
        raise ValueError(f"{', '.join(names)} must share one dtype")
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError(f"{', '.join(names)} must be contiguous")
    if not all(t.is_cuda for t in tensors):
        raise ValueError(f"{', '.join(names)} must be CUDA tensors")


def fold_weight(weight, b, out=None):
    """b_folded[k, n] = weight[k] * b[k, n] on the device (once per weight pair)."""
    import torch

    k, n = b.shape
    if tuple(weight.shape) != (k,):
        raise ValueError(f"weight {tuple(weight.shape)} must have K = {k} elements")
    if out is None:
        out = torch.empty_like(b)
    if tuple(out.shape) != (k, n):
        raise ValueError("out must have b's shape")
    _check((weight, b, out), ("weight", "b", "out"))
    _native.check(
        _native.load().bokt_rmsnorm_fold_weight(weight.data_ptr(), b.data_ptr(), out.data_ptr(),
                                                k, n, _native.dtype_code(b.dtype),
                                                _native.current_stream(b.device)),
        "bokt_rmsnorm_fold_weight",
    )
    return out


def row_scale(x, out, epsilon=1e-6):
    """out[m] = rsqrt(mean(x[m]^2) + epsilon) (fp32, one pass over x)."""
    import torch

    m, k = x.shape
    if out.dtype != torch.float32 or out.numel() != m or not out.is_contiguous():
        raise ValueError("out must be a contiguous fp32 tensor with one entry per row")
    _check((x,), ("x",))
    _native.check(
        _native.load().bokt_rmsnorm_row_scale(x.data_ptr(), out.data_ptr(), m, k, float(epsilon),
                                              _native.dtype_code(x.dtype),
                                              _native.current_stream(x.device)),
        "bokt_rmsnorm_row_scale",
    )


def gemm_row_scaled(a, b, out, scale, params):
    """out[m, :] = scale[m] * (a[m, :] @ b) with the scale applied to the fp32
    accumulator (the GEMM half of ``launch``)."""
    import torch

    m, k = a.shape
    n = b.shape[1]
    if b.shape[0] != k or tuple(out.shape) != (m, n):
        raise ValueError("shape mismatch")
    if scale.dtype != torch.float32 or scale.numel() < m or not scale.is_contiguous():
        raise ValueError("scale must be a contiguous fp32 tensor of at least M entries")
    _check((a, b, out), ("a", "b", "out"))
    p = _native.make_params(params)
    _native.check(
        _native.load().bokt_gemm_row_scaled(a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                            scale.data_ptr(), m, n, k,
                                            _native.dtype_code(a.dtype), ctypes.byref(p),
                                            _native.current_stream(a.device)),
        "bokt_gemm_row_scaled",
    )


def _workspace(device, m):
    import torch

    key = (device.index, m)
    with _lock:
        ws = _row_scale.get(key)
        if ws is None:
            ws = torch.empty(max(m, 1), device=device, dtype=torch.float32)
            _row_scale[key] = ws
        return ws


def launch(x, b_folded, out, params, epsilon=1e-6, scale_workspace=None):
    """out = rmsnorm(x, weight, epsilon) @ b for b_folded = fold_weight(weight, b).

    The per-row factors go to ``scale_workspace`` (fp32 [M]) or to a per-device
    buffer allocated on the first call for this M (make that call before CUDA
    graph capture)."""
    import torch

    m, k = x.shape
    n = b_folded.shape[1]
    if b_folded.shape[0] != k or tuple(out.shape) != (m, n):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, b_folded {tuple(b_folded.shape)}, "
                         f"out {tuple(out.shape)}")
    _check((x, b_folded, out), ("x", "b_folded", "out"))
    if not (math.isfinite(epsilon) and epsilon >= 0):
        raise ValueError("epsilon must be finite and non-negative")
    ws = scale_workspace if scale_workspace is not None else _workspace(x.device, m)
    if ws.dtype != torch.float32 or ws.numel() < m or not ws.is_contiguous():
        raise ValueError("scale_workspace must be a contiguous fp32 tensor of at least M entries")
    lib = _native.load()
    dtype = _native.dtype_code(x.dtype)
    p = _native.make_params(params)
    _native.check(
        lib.bokt_rmsnorm_gemm(x.data_ptr(), b_folded.data_ptr(), out.data_ptr(), ws.data_ptr(), m,
                              n, k, float(epsilon), dtype, ctypes.byref(p),
                              _native.current_stream(x.device)),
        "bokt_rmsnorm_gemm",
    )
    return _native.kernel_attrs(_native.KERNEL_RMSNORM_GEMM, dtype, n, k, params, x.device.index)
