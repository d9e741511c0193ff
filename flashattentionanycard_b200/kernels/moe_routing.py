"""Device-resident MoE routing front end (sm_100a) feeding the grouped GEMM.

The reference builds expert offsets with a host prefix sum
(``bo_kernel_tuner/tuner/worker.py:81-86``) and leaves routing, sorting and
scatter outside the operator (``kernels/moe_grouped_gemm.py:3``).  These
kernels produce, from the flattened top-k expert ids of every token:

* ``counts[E]``     tokens routed to each expert,
* ``offsets[E+1]``  exclusive prefix sum (int32, optionally also int64),
* ``perm[A]``       stable order of assignments by expert (packed row -> assignment),
* ``inv_perm[A]``   combine indices (assignment -> packed row),

bit-identical to ``numpy.argsort(ids, kind="stable")`` / ``bincount`` / ``cumsum``.
``gather_rows`` then packs token activations in expert order for the grouped GEMM.
"""

import ctypes

from flashattentionanycard_b200 import _native


def workspace_bytes(assignments, experts):
    return int(_native.load().bokt_moe_route_workspace_bytes(int(assignments), int(experts)))


def route(expert_ids, num_experts, counts, offsets, perm, inv_perm, workspace, offsets64=None):
    """Launch the routing kernels on the current stream (no sync, no allocation)."""
    import torch

    a = expert_ids.numel()
    for name, tensor, size in (("counts", counts, num_experts), ("offsets", offsets, num_experts + 1),
                               ("perm", perm, a), ("inv_perm", inv_perm, a)):
        if tensor.dtype != torch.int32 or tensor.numel() != size or not tensor.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor of {size} elements")
    if expert_ids.dtype != torch.int32 or not expert_ids.is_contiguous():
        raise ValueError("expert_ids must be a contiguous int32 tensor")
    if offsets64 is not None and (offsets64.dtype != torch.int64 or offsets64.numel() != num_experts + 1):
        raise ValueError("offsets64 must be an int64 tensor of E+1 elements")
    lib = _native.load()
    _native.check(
        lib.bokt_moe_route(
            expert_ids.data_ptr(), a, int(num_experts), counts.data_ptr(), offsets.data_ptr(),
            offsets64.data_ptr() if offsets64 is not None else None, perm.data_ptr(),
            inv_perm.data_ptr(), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
            _native.current_stream(expert_ids.device),
        ),
        "bokt_moe_route",
    )


def gather_rows(src, index, out, divisor=1):
    """out[j] = src[index[j] // divisor] for every row j of out (device kernel)."""
    import torch

    if index.dtype != torch.int32 or index.numel() != out.shape[0]:
        raise ValueError("index must be int32 with one entry per output row")
    if src.dtype != out.dtype or src.shape[1:] != out.shape[1:]:
        raise ValueError("src and out must share dtype and row shape")
    if not (src.is_contiguous() and out.is_contiguous() and index.is_contiguous()):
        raise ValueError("src, index and out must be contiguous")
    cols = 1
    for d in out.shape[1:]:
        cols *= d
    lib = _native.load()
    _native.check(
        lib.bokt_gather_rows(src.data_ptr(), src.shape[0], out.data_ptr(), index.data_ptr(),
                             out.shape[0], cols, out.element_size(), int(divisor),
                             _native.current_stream(out.device)),
        "bokt_gather_rows",
    )


class MoeRouter:
    """Owns the routing outputs and the scratch buffer for one (assignments, experts) shape.

    Buffers are allocated once in the constructor, so ``__call__`` can be
    captured in a CUDA graph."""

    def __init__(self, assignments, experts, device, with_offsets64=False):
        import torch

        self.assignments, self.experts = int(assignments), int(experts)
        i32 = dict(device=device, dtype=torch.int32)
        self.counts = torch.zeros(self.experts, **i32)
        self.offsets = torch.zeros(self.experts + 1, **i32)
        self.offsets64 = (torch.zeros(self.experts + 1, device=device, dtype=torch.int64)
                          if with_offsets64 else None)
        self.perm = torch.zeros(self.assignments, **i32)
        self.inv_perm = torch.zeros(self.assignments, **i32)
        nbytes = max(workspace_bytes(self.assignments, self.experts), 4)
        self.workspace = torch.empty(nbytes // 4, **i32)

    def __call__(self, expert_ids):
        if expert_ids.numel() != self.assignments:
            raise ValueError("expert_ids size differs from the router's shape")
        route(expert_ids.reshape(-1), self.experts, self.counts, self.offsets, self.perm,
              self.inv_perm, self.workspace, self.offsets64)
        return self


def topk_gate(logits, k, ids, gates, renormalize=True):
    """Top-k softmax gate on the device: ids [T, k] int32, gates [T, k] fp32
    (softmax of the logits at the picked experts, renormalised to sum 1 when
    ``renormalize``); ties go to the lower expert index."""
    import torch

    t, e = logits.shape
    codes = {torch.float16: _native.FP16, torch.bfloat16: _native.BF16, torch.float32: 2}
    if logits.dtype not in codes or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous fp16/bf16/fp32 [tokens, experts] tensor")
    if ids.dtype != torch.int32 or tuple(ids.shape) != (t, k) or not ids.is_contiguous():
        raise ValueError("ids must be a contiguous int32 [tokens, k] tensor")
    if gates.dtype != torch.float32 or tuple(gates.shape) != (t, k) or not gates.is_contiguous():
        raise ValueError("gates must be a contiguous fp32 [tokens, k] tensor")
    _native.check(_native.load().bokt_moe_topk_gate(
        logits.data_ptr(), codes[logits.dtype], t, e, int(k), 1 if renormalize else 0,
        ids.data_ptr(), gates.data_ptr(), _native.current_stream(logits.device)),
        "bokt_moe_topk_gate")


def combine(y, gates, out, rows=None):
    """out[t] = sum_j gates[t, j] * y[rows[t*k + j] if rows is given else t*k + j]
    on the device (fp32 accumulation)."""
    import torch

    t, k = gates.shape
    if gates.dtype != torch.float32 or not gates.is_contiguous():
        raise ValueError("gates must be a contiguous fp32 [tokens, k] tensor")
    if y.dtype != out.dtype or y.shape[1] != out.shape[1] or out.shape[0] != t:
        raise ValueError("y [rows, N] and out [tokens, N] must share dtype and N")
    if rows is not None and (rows.dtype != torch.int32 or rows.numel() != t * k):
        raise ValueError("rows must be int32 with tokens * k entries")
    _native.check(_native.load().bokt_moe_combine(
        y.data_ptr(), y.shape[0], rows.data_ptr() if rows is not None else None, gates.data_ptr(),
        out.data_ptr(), t, int(k), y.shape[1], _native.dtype_code(y.dtype),
        _native.current_stream(y.device)), "bokt_moe_combine")
