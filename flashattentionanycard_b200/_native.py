"""ctypes binding of the in-tree C-ABI library ``libbokt_sm100.so`` (include/bokt.h).

The library is the only compute path: there is no Triton, PyTorch or CPU
fallback behind the ``launch`` functions.  A missing or stale library raises
``RuntimeError`` at the first call instead of silently running something else.
"""

import ctypes
import os
import threading
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "libbokt_sm100.so"
ABI_VERSION = 1

FP16, BF16 = 0, 1
KERNEL_GEMM, KERNEL_RMSNORM, KERNEL_MOE_GROUPED_GEMM, KERNEL_RMSNORM_GEMM = 0, 1, 2, 3

BOKT_ERR_CUDA_RC = 4

ERRORS = {
    1: "invalid argument",
    2: "unsupported",
    3: "invalid launch configuration",
    4: "CUDA error",
    5: "device-reported failure",
}

# Public parameter names (search-space keys) -> bokt_params fields.
PARAM_FIELDS = {
    "BLOCK_M": "block_m",
    "BLOCK_N": "block_n",
    "BLOCK_K": "block_k",
    "num_stages": "stages",
    "GROUP_M": "group_m",
    "CTA_MULTIPLIER": "cta_multiplier",
    "num_warps": "num_warps",
    "ROWS_PER_CTA": "rows_per_cta",
    "SPLIT_K": "split_k",
    "CTA_GROUP": "cta_group",
    "RASTER": "raster",
}


class BoktParams(ctypes.Structure):
    _fields_ = [
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("group_m", ctypes.c_int32),
        ("cta_multiplier", ctypes.c_int32),
        ("num_warps", ctypes.c_int32),
        ("rows_per_cta", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("cta_group", ctypes.c_int32),
        ("raster", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 5),
    ]


class BoktAttrs(ctypes.Structure):
    _fields_ = [
        ("shared_bytes", ctypes.c_int32),
        ("registers", ctypes.c_int32),
        ("local_bytes", ctypes.c_int32),
        ("threads", ctypes.c_int32),
        ("max_threads", ctypes.c_int32),
        ("path", ctypes.c_int32),
    ]


_VP, _I32, _I64, _F32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
_PP = ctypes.POINTER(BoktParams)

SIGNATURES = {
    "bokt_abi_version": (_I32, []),
    "bokt_built_sm": (_I32, []),
    "bokt_last_error": (ctypes.c_char_p, []),
    "bokt_gemm": (_I32, [_VP, _VP, _VP, _I32, _I32, _I32, _I32, _PP, _VP]),
    "bokt_rmsnorm": (_I32, [_VP, _VP, _VP, _I32, _I32, _F32, _I32, _PP, _VP]),
    "bokt_rmsnorm_fold_weight": (_I32, [_VP, _VP, _VP, _I32, _I32, _I32, _VP]),
    "bokt_rmsnorm_row_scale": (_I32, [_VP, _VP, _I32, _I32, _F32, _I32, _VP]),
    "bokt_gemm_row_scaled": (_I32, [_VP, _VP, _VP, _VP, _I32, _I32, _I32, _I32, _PP, _VP]),
    "bokt_rmsnorm_gemm": (_I32, [_VP, _VP, _VP, _VP, _I32, _I32, _I32, _F32, _I32, _PP, _VP]),
    "bokt_moe_grouped_gemm": (
        _I32,
        [_VP, _VP, _VP, _I32, _VP, _I32, _I32, _I32, _I32, _I32, _I32, _PP, _VP],
    ),
    "bokt_gemm_ex": (_I32, [_VP, _VP, _VP, _I32, _I32, _I32, _I32, _PP, _VP, _I64, _VP]),
    "bokt_gemm_workspace_bytes": (_I64, [_I32, _PP]),
    "bokt_splitk_schedule": (_I32, [_I32, _I32, _I32, _I32, _VP, _I32]),
    "bokt_splitk_reduce_sources": (_I32, [_I32, _I32, _I32, _I32, _VP, _I32]),
    "bokt_moe_grouped_gemm_ex": (
        _I32,
        [_VP, _VP, _VP, _I32, _VP, _I32, _I32, _I32, _I32, _I32, _I32, _PP, _VP, _I64, _VP],
    ),
    "bokt_moe_route_workspace_bytes": (_I64, [_I32, _I32]),
    "bokt_moe_route": (_I32, [_VP, _I32, _I32, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _VP]),
    "bokt_moe_route_noalloc_max_words": (_I64, []),
    "bokt_moe_route_noalloc": (_I32, [_VP, _I32, _I32, _VP, _VP, _VP, _VP, _VP, _VP]),
    "bokt_gather_rows": (_I32, [_VP, _I64, _VP, _VP, _I32, _I32, _I32, _I32, _VP]),
    "bokt_gather_rows_indirect": (
        _I32, [_VP, _I64, _VP, _VP, _I64, _VP, _I32, _I32, _I32, _I32, _I64, _VP]),
    "bokt_ep_keys": (_I32, [_VP] * 8 + [_I32] * 7 + [_VP] * 4),
    "bokt_check_counts": (_I32, [_VP, _VP, _I32, _I32, _VP]),
    "bokt_moe_grouped_gemm_scatter": (
        _I32, [_VP, _VP, _VP, _I32] + [_I32] * 6 + [_VP, _VP, _I32, _I32, _PP, _VP]),
    "bokt_ep_plan": (_I32, [_VP, _VP, _VP, _I32, _VP, _I32, _I32, _I32] + [_VP] * 6 + [_VP]),
    "bokt_ep_dispatch": (_I32, [_VP, _I32, _I32] + [_VP] * 11 + [_I32] * 4 + [_VP]),
    "bokt_ep_rowmap": (_I32, [_VP] * 9 + [_I32] * 4 + [_VP, _VP]),
    "bokt_ep_put": (_I32, [_VP, _I64, _VP, _I64, _I32, _VP]),
    "bokt_ep_barrier": (_I32, [_VP, _VP, _I32, _I32, _I64, _VP]),
    "bokt_ep_barrier_combine": (
        _I32, [_VP, _VP, _I32, _I32, _I64, _VP, _VP, _VP, _I32, _I32, _I32, _I32, _VP]),
    "bokt_ipc_export": (_I32, [_VP, _VP, ctypes.POINTER(ctypes.c_int64)]),
    "bokt_ipc_import": (_I32, [_VP, _I64, ctypes.POINTER(_VP), ctypes.POINTER(_VP)]),
    "bokt_ipc_close": (_I32, [_VP]),
    "bokt_selftest_bounded_wait": (_I32, [_I64, _VP, _VP]),
    "bokt_moe_topk_gate": (_I32, [_VP, _I32, _I32, _I32, _I32, _I32, _VP, _VP, _VP]),
    "bokt_moe_combine": (_I32, [_VP, _I64, _VP, _VP, _VP, _I32, _I32, _I32, _I32, _VP]),
    "bokt_kernel_attrs": (
        _I32,
        [_I32, _I32, _I32, _I32, _PP, ctypes.POINTER(BoktAttrs)],
    ),
    "bokt_device_status": (
        _I32,
        [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), _I32],
    ),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the ctypes library; raise RuntimeError if absent."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("BOKT_LIBRARY", LIBRARY_PATH))
        if not path.exists():
            raise RuntimeError(
                f"sm_100a kernel library not built: {path} is missing "
                "(run `make -C flashattentionanycard_b200/csrc` or __graft_entry__.build())"
            )
        lib = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.bokt_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{path}: ABI version {lib.bokt_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def check(rc, what):
    """Turn a non-zero status into RuntimeError carrying bokt_last_error()."""
    if rc != 0:
        message = load().bokt_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({ERRORS.get(rc, rc)}): {message}")


def make_params(params):
    """Convert a search-space parameter dict to bokt_params (unknown keys rejected)."""
    p = BoktParams()
    for key, value in (params or {}).items():
        field = PARAM_FIELDS.get(key)
        if field is None:
            raise ValueError(f"Unknown launch parameter {key!r}")
        if type(value) is not int:
            raise ValueError(f"Launch parameter {key} must be int, got {type(value).__name__}")
        setattr(p, field, value)
    return p


def dtype_code(dtype):
    import torch

    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float16:
        return FP16
    raise ValueError(f"Unsupported dtype {dtype}; expected float16 or bfloat16")


def current_stream(device):
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def device_status(reset=True):
    """Return (code, detail) of the device status word (synchronises the device)."""
    lib = load()
    code, detail = ctypes.c_int(0), ctypes.c_int(0)
    check(lib.bokt_device_status(ctypes.byref(code), ctypes.byref(detail), 1 if reset else 0),
          "bokt_device_status")
    return code.value, detail.value


class _Metadata:
    def __init__(self, shared):
        self.shared = shared


class CompiledKernel:
    """What ``launch`` returns: the fields the worker reads from Triton's
    compiled-kernel object (tuner/worker.py:193,203-204 of the reference):
    ``metadata.shared``, ``n_regs`` and ``n_spills``.  ``n_spills`` is the
    kernel's local memory per thread in 4-byte words (0 when nothing spills)."""

    def __init__(self, attrs):
        self.metadata = _Metadata(int(attrs.shared_bytes))
        self.n_regs = int(attrs.registers)
        self.n_spills = int(attrs.local_bytes) // 4
        self.threads = int(attrs.threads)
        self.path = {0: "tcgen05", 1: "tcgen05_edge", 2: "vector", 3: "scalar", 4: "ring",
                     5: "pipelined"}.get(attrs.path, "?")


_splitk_ws = {}


def splitk_workspace(kernel, params, device):
    """(pointer, bytes) of the split-K workspace for ``params`` on ``device``
    ((None, 0) when SPLIT_K <= 1).

    One zero-filled buffer per device, allocated on the first split-K call
    (that first call must come before any graph capture, as the reference's
    warm-up calls do) and kept for the life of the process; it grows only if a
    later configuration needs more.  Calls that share it must not overlap on
    the GPU: the library keeps a launch sequence number in it."""
    import torch

    if int((params or {}).get("SPLIT_K", 1)) <= 1:
        return None, 0
    lib = load()
    p = make_params(params)
    need = int(lib.bokt_gemm_workspace_bytes(kernel, ctypes.byref(p)))
    if need < 0:
        check(BOKT_ERR_CUDA_RC, "bokt_gemm_workspace_bytes")
    key = device if isinstance(device, int) else torch.device(device).index
    buf = _splitk_ws.get(key)
    if buf is None or buf.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("split-K workspace must be allocated before graph capture: "
                               "make one uncaptured call with these parameters first")
        buf = torch.zeros(need, dtype=torch.uint8, device=torch.device("cuda", key))
        _splitk_ws[key] = buf
    return ctypes.c_void_p(buf.data_ptr()), buf.numel()


def splitk_schedule(ntiles, split_k, nkb, launched):
    """Segments of the split-K schedule, computed by the library's own host
    copy of the device arithmetic: list of (worker, tile, kb0, kb1,
    first_contributor, contributors)."""
    lib = load()
    n = lib.bokt_splitk_schedule(ntiles, split_k, nkb, launched, None, 0)
    if n < 0:
        raise RuntimeError(lib.bokt_last_error().decode())
    buf = (ctypes.c_int32 * (6 * max(n, 1)))()
    lib.bokt_splitk_schedule(ntiles, split_k, nkb, launched, buf, n)
    return [tuple(buf[6 * i:6 * i + 6]) for i in range(n)]


def splitk_reduce_sources(ntiles, split_k, nkb, launched):
    """Partials the separate split-K reduction adds, in its order: list of
    (tile, worker, which) -- workspace slot 2 c + which of worker CTA slot c."""
    lib = load()
    n = lib.bokt_splitk_reduce_sources(ntiles, split_k, nkb, launched, None, 0)
    if n < 0:
        raise RuntimeError(lib.bokt_last_error().decode())
    buf = (ctypes.c_int32 * (3 * max(n, 1)))()
    lib.bokt_splitk_reduce_sources(ntiles, split_k, nkb, launched, buf, n)
    return [tuple(buf[3 * i:3 * i + 3]) for i in range(n)]


_attr_cache = {}


def kernel_attrs(kernel, dtype, n, k, params, device):
    key = (kernel, dtype, n, k, tuple(sorted((params or {}).items())), device)
    hit = _attr_cache.get(key)
    if hit is None:
        lib = load()
        attrs = BoktAttrs()
        p = make_params(params)
        check(lib.bokt_kernel_attrs(kernel, dtype, n, k, ctypes.byref(p), ctypes.byref(attrs)),
              "bokt_kernel_attrs")
        hit = _attr_cache[key] = CompiledKernel(attrs)
    return hit
