"""One persistent launch for ragged experts with packed tokens and shared N/K (sm_100a).

Drop-in for the reference's ``bo_kernel_tuner/kernels/moe_grouped_gemm.py:61-65``:
``launch(x, weights, offsets, out, params, sm_count)`` computes, for every
expert e, ``out[off[e]:off[e+1]] = x[off[e]:off[e+1]] @ weights[e]`` with
``weights`` of shape [E, K, N].  ``offsets`` (E+1 entries, int64 as the
reference's worker builds them, or int32 as the routing kernels produce them)
stays on the device and is read by the kernel.  Empty experts cost nothing,
every output tile has exactly one writer, and the persistent grid is
``sm_count * CTA_MULTIPLIER`` CTAs as in the reference.  ``SPLIT_K`` > 1
(single-CTA tiles) splits every tile's K loop across CTAs, with the fp32
partials in a per-device workspace allocated on the first such call.

Routing, sorting and scatter stay outside this operator, as in the reference
(``moe_grouped_gemm.py:3``); the device routing front end lives in
``kernels/moe_routing.py``.
"""

import ctypes

from flashattentionanycard_b200 import _native


def launch(x, weights, offsets, out, params, sm_count):
    import torch

    e, k, n = weights.shape
    t = x.shape[0]
    if x.shape[1] != k or tuple(out.shape) != (t, n):
        raise ValueError(
            f"shape mismatch: x {tuple(x.shape)}, weights {tuple(weights.shape)}, out {tuple(out.shape)}"
        )
    if tuple(offsets.shape) != (e + 1,):
        raise ValueError(f"offsets must have E+1 = {e + 1} entries, got {tuple(offsets.shape)}")
    if offsets.dtype not in (torch.int32, torch.int64):
        raise ValueError("offsets must be int32 or int64")
    if not (x.dtype == weights.dtype == out.dtype):
        raise ValueError("x, weights and out must share one dtype")
    tensors = (x, weights, offsets, out)
    if not all(v.is_contiguous() for v in tensors):
        raise ValueError("x, weights, offsets and out must be contiguous")
    if not all(v.is_cuda for v in tensors):
        raise ValueError("x, weights, offsets and out must be CUDA tensors")
    lib = _native.load()
    dtype = _native.dtype_code(x.dtype)
    p = _native.make_params(params)
    ws, ws_bytes = _native.splitk_workspace(_native.KERNEL_MOE_GROUPED_GEMM, params, x.device)
    _native.check(
        lib.bokt_moe_grouped_gemm_ex(
            x.data_ptr(), weights.data_ptr(), offsets.data_ptr(),
            1 if offsets.dtype == torch.int64 else 0, out.data_ptr(), t, e, n, k, dtype,
            int(sm_count), ctypes.byref(p), ws, ws_bytes, _native.current_stream(x.device),
        ),
        "bokt_moe_grouped_gemm",
    )
    # The library takes the edge kernel for any operand not 16-byte aligned;
    # report that kernel's attributes then (k = 1 selects it in the query).
    aligned = all(t.data_ptr() % 16 == 0 for t in (x, weights, out))
    return _native.kernel_attrs(_native.KERNEL_MOE_GROUPED_GEMM, dtype, n, k if aligned else 1,
                                params, x.device.index)
