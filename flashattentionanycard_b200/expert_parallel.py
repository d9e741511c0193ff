"""Expert-parallel MoE grouped GEMM across GPUs (one process per GPU, NCCL).

The reference runs one GPU only; this is the multi-GPU form of its grouped GEMM
(``kernels/moe_grouped_gemm.py``) for the 64-expert, top-2, Zipf-routed case.

Layout: tokens are owned in contiguous blocks of ``tokens_per_rank`` per rank
(rank r owns tokens [r*T/G, (r+1)*T/G)).  Experts are served by *virtual
experts*: expert e gets ``replicas[e]`` of them, which split the expert's packed
rows contiguously (packed row q of the expert goes to replica q*R_e // c_e), so
a hot expert is spread over several GPUs without splitting any row or column;
every assignment row crosses NVLink once on dispatch and once on combine.
Virtual experts are packed onto ranks with longest-processing-time-first.  The
placement is a deterministic function of the global expert counts, so every
rank derives the same plan and the result is bit-identical to the one-GPU
routing.

One step (every rank, same order of collectives):
  1. all-gather the int32 expert ids of all tokens (NCCL, 4 * T * topk bytes);
  2. global routing on every rank (bokt_moe_route): counts, offsets, perm;
  3. per-row keys (bokt_ep_keys) and three stable counting sorts: the send
     order (by destination), the receive order (by source) and the local
     grouped-GEMM order (by local virtual expert, which also gives its offsets);
  4. the sort sizes are checked against the plan on the device
     (bokt_check_counts); the NCCL split sizes come from the plan, so the step
     needs no host synchronisation;
  5. gather the rows to send (bokt_gather_rows_indirect), all_to_all_single;
  6. reorder received rows into local expert order, grouped GEMM (tcgen05);
  7. gather result rows back in receive order, all_to_all_single back;
  8. reorder into local assignment order (token-major, topk slots).
"""

import ctypes
from dataclasses import dataclass, field

import numpy as np

from flashattentionanycard_b200 import _native


# ----------------------------------------------------------------------------- planning
@dataclass
class Placement:
    world: int
    experts: int
    replicas: np.ndarray  # int32 [E]
    vbase: np.ndarray  # int32 [E]
    v_expert: np.ndarray  # int32 [V]
    v_replica: np.ndarray  # int32 [V]
    v_rows: np.ndarray  # int64 [V] packed rows served
    v_rank: np.ndarray  # int32 [V]
    v_local: np.ndarray  # int32 [V] index among the rank's virtual experts
    local: list = field(default_factory=list)  # per rank: ascending list of v
    rank_rows: np.ndarray = None  # int64 [world] rows served per rank

    @property
    def virtual_experts(self):
        return int(self.v_expert.size)


def replica_rows(count, replicas):
    """Rows of each replica when ``count`` packed rows are split so that row q
    goes to replica q * replicas // count (bokt_ep_keys)."""
    bounds = [-(-j * count // replicas) for j in range(replicas + 1)]  # ceil(j c / R)
    return np.diff(np.asarray(bounds, dtype=np.int64))


def plan_placement(counts, world, cap_fraction=0.25):
    """Deterministic virtual-expert placement for ``world`` ranks.

    Each expert gets R_e = ceil(c_e / cap) replicas with cap = cap_fraction *
    total / world (R_e = 1 on one rank), then replicas are placed largest
    first on the least-loaded rank (ties: lower rank).  The LPT bound keeps the
    busiest rank within cap of the average."""
    counts = np.asarray(counts, dtype=np.int64)
    experts = counts.size
    total = int(counts.sum())
    if world < 1:
        raise ValueError("world must be >= 1")
    if world == 1:
        replicas = np.ones(experts, dtype=np.int64)
    else:
        cap = max(1, -(-int(total * cap_fraction) // world))
        replicas = np.maximum(1, -(-counts // cap))
        replicas = np.minimum(replicas, world * 4)
    vbase = np.concatenate([[0], np.cumsum(replicas)[:-1]]).astype(np.int64)
    v_expert, v_replica, v_rows = [], [], []
    for e in range(experts):
        rows = replica_rows(int(counts[e]), int(replicas[e])) if counts[e] else np.zeros(
            int(replicas[e]), np.int64)
        for j in range(int(replicas[e])):
            v_expert.append(e)
            v_replica.append(j)
            v_rows.append(int(rows[j]))
    v_expert = np.asarray(v_expert, dtype=np.int32)
    v_replica = np.asarray(v_replica, dtype=np.int32)
    v_rows = np.asarray(v_rows, dtype=np.int64)
    order = sorted(range(v_rows.size), key=lambda v: (-int(v_rows[v]), v))
    load = np.zeros(world, dtype=np.int64)
    v_rank = np.zeros(v_rows.size, dtype=np.int32)
    for v in order:
        r = int(np.argmin(load))  # first minimum: lowest rank on ties
        v_rank[v] = r
        load[r] += v_rows[v]
    local = [sorted(int(v) for v in np.nonzero(v_rank == r)[0]) for r in range(world)]
    v_local = np.zeros(v_rows.size, dtype=np.int32)
    for r in range(world):
        for i, v in enumerate(local[r]):
            v_local[v] = i
    return Placement(world, experts, replicas.astype(np.int32), vbase.astype(np.int32), v_expert,
                     v_replica, v_rows, v_rank, v_local, local, load)


@dataclass
class Plan:
    """Per-rank split sizes implied by a routing table and a placement."""

    send: np.ndarray  # int64 [world, world]: rows rank r sends to rank d
    local_rows: list  # per rank: int64 [n_local] rows per local virtual expert

    def recv(self, rank):
        return self.send[:, rank]


def row_destinations(ids_flat, placement, topk, tokens_per_rank):
    """(perm, owner[p], dest[p], v[p]) of every packed row of the global routing."""
    ids_flat = np.asarray(ids_flat, dtype=np.int64)
    e_count = np.bincount(ids_flat, minlength=placement.experts)
    offsets = np.concatenate([[0], np.cumsum(e_count)])
    perm = np.argsort(ids_flat, kind="stable")
    e = ids_flat[perm]
    q = np.arange(perm.size) - offsets[e]
    reps = placement.replicas.astype(np.int64)[e]
    j = np.where(e_count[e] > 0, (q * reps) // np.maximum(e_count[e], 1), 0)
    v = placement.vbase.astype(np.int64)[e] + j
    dest = placement.v_rank.astype(np.int64)[v]
    owner = (perm // topk) // tokens_per_rank
    return perm, owner, dest, v


def plan_splits(ids_flat, placement, topk, tokens_per_rank):
    world = placement.world
    _, owner, dest, v = row_destinations(ids_flat, placement, topk, tokens_per_rank)
    send = np.zeros((world, world), dtype=np.int64)
    np.add.at(send, (owner, dest), 1)
    local_rows = []
    for r in range(world):
        lv = placement.v_local.astype(np.int64)[v[dest == r]]
        local_rows.append(np.bincount(lv, minlength=len(placement.local[r])).astype(np.int64))
    return Plan(send, local_rows)


# ----------------------------------------------------------------------------- device step
class ExpertParallelMoE:
    """One rank of the expert-parallel grouped GEMM.

    ``local_weights``: [n_local, K, N] weights of this rank's virtual experts in
    ``placement.local[rank]`` order (W[v_expert[v]]).  ``plan``: split sizes for
    the routing the step will see; the step verifies them on the device."""

    def __init__(self, local_weights, placement, plan, rank, world, topk, tokens_per_rank,
                 group=None, params=None, sm_count=None):
        import torch

        from flashattentionanycard_b200.kernels.moe_routing import MoeRouter

        self.rank, self.world, self.topk = rank, world, topk
        self.tokens_per_rank = tokens_per_rank
        self.group = group
        self.params = dict(params or {})
        self.w = local_weights
        self.device = local_weights.device
        dev = self.device
        self.k, self.n = int(local_weights.shape[1]), int(local_weights.shape[2])
        self.n_local = len(placement.local[rank])
        if local_weights.shape[0] != self.n_local:
            raise ValueError("local_weights must hold one [K, N] slice per local virtual expert")
        self.sm = sm_count or torch.cuda.get_device_properties(dev).multi_processor_count
        self.experts = placement.experts
        self.a_global = tokens_per_rank * world * topk
        self.a_local = tokens_per_rank * topk
        i32 = dict(device=dev, dtype=torch.int32)
        self.replicas = torch.tensor(placement.replicas, **i32)
        self.vbase = torch.tensor(placement.vbase, **i32)
        self.v_rank = torch.tensor(placement.v_rank, **i32)
        self.v_local = torch.tensor(placement.v_local, **i32)
        self.ids_global = torch.zeros(self.a_global, **i32)
        self.route_global = MoeRouter(self.a_global, self.experts, dev)
        self.route_send = MoeRouter(self.a_global, world + 1, dev)
        self.route_recv = MoeRouter(self.a_global, world + 1, dev)
        self.route_local = MoeRouter(self.a_global, self.n_local + 1, dev)
        self.key_send = torch.zeros(self.a_global, **i32)
        self.key_recv = torch.zeros(self.a_global, **i32)
        self.key_local = torch.zeros(self.a_global, **i32)
        self.send_sizes = [int(v) for v in plan.send[rank]]
        self.recv_sizes = [int(v) for v in plan.recv(rank)]
        self.n_send, self.n_recv = sum(self.send_sizes), sum(self.recv_sizes)
        local_rows = plan.local_rows[rank]
        self.expected_send = torch.tensor(self.send_sizes, **i32)
        self.expected_recv = torch.tensor(self.recv_sizes, **i32)
        self.expected_local = torch.tensor([int(v) for v in local_rows], **i32)
        if int(local_rows.sum()) != self.n_recv:
            raise ValueError("plan is inconsistent: local rows != received rows")
        dt = local_weights.dtype
        self.send_x = torch.empty(max(self.n_send, 1), self.k, device=dev, dtype=dt)
        self.recv_x = torch.empty(max(self.n_recv, 1), self.k, device=dev, dtype=dt)
        self.x_packed = torch.empty(max(self.n_recv, 1), self.k, device=dev, dtype=dt)
        self.y_packed = torch.empty(max(self.n_recv, 1), self.n, device=dev, dtype=dt)
        self.y_send = torch.empty(max(self.n_recv, 1), self.n, device=dev, dtype=dt)
        self.y_ret = torch.empty(max(self.n_send, 1), self.n, device=dev, dtype=dt)
        self.out = torch.empty(self.a_local, self.n, device=dev, dtype=dt)

    # -- collectives (NCCL on GPU ranks) -------------------------------------------------
    def _all_gather_ids(self, ids_local):
        import torch.distributed as dist

        if self.world == 1:
            self.ids_global.copy_(ids_local.reshape(-1))
        else:
            dist.all_gather_into_tensor(self.ids_global, ids_local.reshape(-1), group=self.group)

    def _all_to_all(self, out, inp, out_sizes, in_sizes):
        import torch.distributed as dist

        if self.world == 1:
            if out_sizes[0]:
                out[: out_sizes[0]].copy_(inp[: in_sizes[0]])
            return
        dist.all_to_all_single(out[: sum(out_sizes)], inp[: sum(in_sizes)],
                               output_split_sizes=out_sizes, input_split_sizes=in_sizes,
                               group=self.group)

    # -- phases ----------------------------------------------------------------------------
    def route(self):
        """Global routing of self.ids_global, keys, the three orders, plan check."""
        lib = _native.load()
        stream = _native.current_stream(self.device)
        g = self.route_global(self.ids_global)
        _native.check(lib.bokt_ep_keys(
            g.perm.data_ptr(), self.ids_global.data_ptr(), g.offsets.data_ptr(),
            g.counts.data_ptr(), self.replicas.data_ptr(), self.vbase.data_ptr(),
            self.v_rank.data_ptr(), self.v_local.data_ptr(), self.a_global, self.experts,
            self.topk, self.tokens_per_rank, self.rank, self.world, self.n_local,
            self.key_send.data_ptr(), self.key_recv.data_ptr(), self.key_local.data_ptr(),
            stream), "bokt_ep_keys")
        self.route_send(self.key_send)
        self.route_recv(self.key_recv)
        self.route_local(self.key_local)
        for tag, (counts, expected) in enumerate(
                ((self.route_send.counts, self.expected_send),
                 (self.route_recv.counts, self.expected_recv),
                 (self.route_local.counts, self.expected_local))):
            n = expected.numel()
            if n:
                _native.check(lib.bokt_check_counts(counts.data_ptr(), expected.data_ptr(), n,
                                                    tag + 1, stream), "bokt_check_counts")

    def _gather(self, src, dst, rows, inner, outer, divisor=1, base=0):
        if rows == 0:
            return
        lib = _native.load()
        _native.check(lib.bokt_gather_rows_indirect(
            src.data_ptr(), src.shape[0], dst.data_ptr(), inner.data_ptr(), inner.numel(),
            outer.data_ptr() if outer is not None else None, rows, src.shape[1],
            src.element_size(), divisor, base, _native.current_stream(self.device)),
            "bokt_gather_rows_indirect")

    def pack_send(self, x_local):
        """send_x[i] = x of the token of the i-th row this rank sends (by destination)."""
        g = self.route_global
        self._gather(x_local, self.send_x, self.n_send, g.perm, self.route_send.perm,
                     divisor=self.topk, base=self.rank * self.tokens_per_rank)

    def unpack_recv(self):
        """x_packed = received rows in local virtual-expert order."""
        self._gather(self.recv_x, self.x_packed, self.n_recv, self.route_recv.inv_perm,
                     self.route_local.perm)

    def compute(self):
        """Grouped GEMM over the local virtual experts (tcgen05)."""
        from flashattentionanycard_b200.kernels import moe_grouped_gemm

        if self.n_recv == 0:
            return
        offsets = self.route_local.offsets[: self.n_local + 1]
        moe_grouped_gemm.launch(self.x_packed[: self.n_recv], self.w, offsets,
                                self.y_packed[: self.n_recv], self.params, self.sm)

    def pack_return(self):
        """y_send = result rows in receive order (grouped by token owner)."""
        self._gather(self.y_packed, self.y_send, self.n_recv, self.route_local.inv_perm,
                     self.route_recv.perm)

    def unpack_return(self):
        """out = returned rows in local assignment order (token-major, topk slots)."""
        g = self.route_global
        outer = g.inv_perm[self.rank * self.a_local:(self.rank + 1) * self.a_local]
        self._gather(self.y_ret, self.out, self.a_local, self.route_send.inv_perm, outer)
        return self.out

    def forward(self, x_local, ids_local):
        """x_local [tokens_per_rank, K], ids_local [tokens_per_rank, topk] int32 ->
        [tokens_per_rank * topk, N]: row t*topk + k = x[t] @ W[ids[t, k]]."""
        self._all_gather_ids(ids_local)
        self.route()
        self.pack_send(x_local)
        self._all_to_all(self.recv_x, self.send_x, self.recv_sizes, self.send_sizes)
        self.unpack_recv()
        self.compute()
        self.pack_return()
        self._all_to_all(self.y_ret, self.y_send, self.send_sizes, self.recv_sizes)
        return self.unpack_return()


def local_weight_slices(placement, rank):
    """Global expert index of each local virtual expert of ``rank``."""
    return [int(placement.v_expert[v]) for v in placement.local[rank]]


# ----------------------------------------------------------------------------- peer-memory step
def _ptr_array(ptrs, device):
    import torch

    return torch.tensor([int(p) for p in ptrs], dtype=torch.int64, device=device)


STATUS_MEANING = {
    1: "a bounded wait timed out (detail: where; 4000 + r = expert-parallel barrier, rank r)",
    2: "an expert id outside [0, E)",
    3: "routing differs from the planned split sizes",
    4: "a rank's packed buffer is too small for this step's routing",
}


def check_device_status(what):
    """Raise RuntimeError if a kernel recorded a failure (synchronises the device)."""
    code, detail = _native.device_status(reset=True)
    if code:
        raise RuntimeError(f"{what}: device status {code} ({STATUS_MEANING.get(code, '?')}), "
                           f"detail {detail}")


class PeerExpertParallelMoE:
    """One rank of the expert-parallel grouped GEMM with dispatch and combine
    over NVLink peer memory instead of NCCL all-to-all.

    Each rank exports (CUDA IPC) its packed-input, output, routing-id and
    barrier-flag buffers and maps the other ranks'.  A step (``sync="device"``):

      1. bokt_ep_put: this rank's expert ids are stored into every rank's copy
         of the global id table, then bokt_ep_barrier;
      2. global routing (bokt_moe_route) and the per-step layout (bokt_ep_plan):
         where each virtual expert's rows live on its rank;
      3. bokt_ep_rowmap: the owner row of every row this rank will compute;
      4. bokt_ep_dispatch: each token row is stored straight into the serving
         rank's packed buffer (NVLink stores), then bokt_ep_barrier;
      5. bokt_moe_grouped_gemm_scatter: the tcgen05 grouped GEMM whose epilogue
         stores every result row into its token owner's output buffer (NVLink
         stores, overlapped with the remaining tiles), then bokt_ep_barrier.

    Every phase is a kernel of this library and the barriers are device-side
    (epochs in device memory, bounded waits), so the step has no host
    collective, no host synchronisation and can be captured in a CUDA graph.
    No row gathers and no all-to-all: every row crosses NVLink once each way,
    written by the kernel that produced it.  ``sync="nccl"`` keeps the NCCL
    all-gather and one-word all-reduce barriers instead.

    Capacity: by default (``capacity="worst"``) each rank's packed buffer holds
    every assignment of the step, so any routing fits whatever plan the
    placement came from.  ``capacity="plan"`` sizes it from ``plan`` (less
    memory); a step whose routing puts more rows on a rank then records
    status 4 and drops those rows, which ``forward(..., check=True)`` turns
    into an exception."""

    def __init__(self, local_weights, placement, plan, rank, world, topk, tokens_per_rank,
                 group=None, params=None, sm_count=None, exchange=True, sync=None,
                 capacity="worst", barrier_timeout_s=5.0):
        """``exchange=False`` skips the IPC pointer exchange: the caller sets the
        per-rank pointers with ``set_peer_pointers`` (ranks sharing one process,
        which drive the phases themselves: ``sync`` defaults to "none")."""
        import torch

        from flashattentionanycard_b200.kernels.moe_routing import MoeRouter

        lib = _native.load()
        if sync is None:
            sync = "device" if exchange else "none"
        if sync not in ("device", "nccl", "none"):
            raise ValueError("sync must be 'device', 'nccl' or 'none'")
        if capacity not in ("worst", "plan"):
            raise ValueError("capacity must be 'worst' or 'plan'")
        self.sync = sync
        self.barrier_timeout_ns = int(barrier_timeout_s * 1e9)
        self.rank, self.world, self.topk = rank, world, topk
        self.tokens_per_rank = tokens_per_rank
        self.group = group
        self.params = _native.make_params(params or {})
        self.w = local_weights
        self.device = dev = local_weights.device
        self.k, self.n = int(local_weights.shape[1]), int(local_weights.shape[2])
        self.n_local = len(placement.local[rank])
        if local_weights.shape[0] != self.n_local:
            raise ValueError("local_weights must hold one [K, N] slice per local virtual expert")
        if self.n_local == 0:
            raise ValueError("every rank must serve at least one virtual expert")
        self.sm = sm_count or torch.cuda.get_device_properties(dev).multi_processor_count
        self.dtype = _native.dtype_code(local_weights.dtype)
        self.experts = placement.experts
        self.V = placement.virtual_experts
        self.a_global = tokens_per_rank * world * topk
        self.a_local = tokens_per_rank * topk
        i32 = dict(device=dev, dtype=torch.int32)
        self.replicas = torch.tensor(placement.replicas, **i32)
        self.vbase = torch.tensor(placement.vbase, **i32)
        self.v_rank = torch.tensor(placement.v_rank, **i32)
        if capacity == "worst":
            caps = [self.a_global] * world
        else:
            caps = [int(plan.local_rows[r].sum()) for r in range(world)]
        self.capacity_rows = caps
        self.capacity = torch.tensor(caps, **i32)
        self.ids_global = torch.zeros(self.a_global, **i32)
        self.route_global = MoeRouter(self.a_global, self.experts, dev)
        self.v_plo = torch.zeros(self.V, **i32)
        self.v_size = torch.zeros(self.V, **i32)
        self.v_lbase = torch.zeros(self.V, **i32)
        self.loffs = torch.zeros(self.n_local + 1, **i32)
        self.rank_rows = torch.zeros(world, **i32)
        cap_me = max(caps[rank], 1)
        self.rowmap = torch.zeros(cap_me, **i32)
        dt = local_weights.dtype
        self.x_packed = torch.zeros(cap_me, self.k, device=dev, dtype=dt)
        self.out = torch.zeros(self.a_local, self.n, device=dev, dtype=dt)
        self.barrier_word = torch.zeros(1, **i32)
        # Device barrier: flags[s] = last epoch rank s signalled to this rank;
        # epoch = [barriers this rank has passed, CTA count of the combining
        # barrier] (zero at start).
        self.sync_flags = torch.zeros(world, **i32)
        self.epoch = torch.zeros(2, **i32)
        # Token-order result of the combine: final[t] = sum_j g[t, j] out[t topk + j].
        self.final = torch.empty(tokens_per_rank, self.n, device=dev, dtype=dt)
        self._own_flag_ptrs = _ptr_array([self.sync_flags.data_ptr()], dev)
        self._peer_bases = {}
        if exchange:
            self.set_peer_pointers(*self._exchange_pointers(lib))

    def shared_buffers(self):
        """The buffers peers write into, in pointer-exchange order."""
        return (self.x_packed, self.out, self.ids_global, self.sync_flags)

    def set_peer_pointers(self, xpk, outs, ids=None, flags=None):
        """Per-rank device pointers of the packed-input, output, id-table and
        barrier-flag buffers (the last two only for ``sync="device"``)."""
        if len(xpk) != self.world or len(outs) != self.world:
            raise ValueError("one pointer per rank")
        self.xpk_ptrs = _ptr_array(xpk, self.device)
        self.out_ptrs = _ptr_array(outs, self.device)
        if ids is not None:
            self.ids_ptrs = _ptr_array(ids, self.device)
        if flags is not None:
            self.flag_ptrs = _ptr_array(flags, self.device)

    def _exchange_pointers(self, lib):
        """Per-rank device pointers of every rank's shared buffers."""
        import torch.distributed as dist

        mine = []
        for t in self.shared_buffers():
            handle = ctypes.create_string_buffer(64)
            offset = ctypes.c_int64(0)
            if self.world > 1:
                _native.check(lib.bokt_ipc_export(t.data_ptr(), handle, ctypes.byref(offset)),
                              "bokt_ipc_export")
            mine.append((bytes(handle.raw), int(offset.value)))
        every = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(every, mine, group=self.group)
        else:
            every = [mine]
        per_buffer = [[] for _ in self.shared_buffers()]
        for r in range(self.world):
            for i, t in enumerate(self.shared_buffers()):
                if r == self.rank:
                    per_buffer[i].append(t.data_ptr())
                    continue
                handle, offset = every[r][i]
                base = self._peer_bases.get(handle)
                if base is None:  # open each peer allocation once
                    b, p = ctypes.c_void_p(), ctypes.c_void_p()
                    _native.check(lib.bokt_ipc_import(handle, 0, ctypes.byref(b),
                                                      ctypes.byref(p)), "bokt_ipc_import")
                    base = self._peer_bases[handle] = b.value
                per_buffer[i].append(base + offset)
        return per_buffer

    def close(self):
        """Unmap the peers' buffers (after the last step has completed everywhere)."""
        lib = _native.load()
        for base in self._peer_bases.values():
            lib.bokt_ipc_close(base)
        self._peer_bases = {}

    def _barrier(self):
        if self.world == 1 or self.sync == "none":
            return
        if self.sync == "nccl":
            import torch.distributed as dist

            dist.all_reduce(self.barrier_word, group=self.group)
            return
        _native.check(_native.load().bokt_ep_barrier(
            self.flag_ptrs.data_ptr(), self.epoch.data_ptr(), self.world, self.rank,
            self.barrier_timeout_ns, _native.current_stream(self.device)), "bokt_ep_barrier")

    def _all_gather_ids(self, ids_local):
        if self.world == 1:
            self.ids_global.copy_(ids_local.reshape(-1))
            return
        if self.sync == "nccl":
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.ids_global, ids_local.reshape(-1), group=self.group)
            return
        if self.sync == "none":
            raise RuntimeError("sync='none': the caller fills ids_global and orders the phases")
        flat = ids_local.reshape(-1)
        if flat.numel() != self.a_local or not flat.is_contiguous() or flat.dtype != self.ids_global.dtype:
            raise ValueError("ids_local must be a contiguous int32 [tokens_per_rank, topk] tensor")
        _native.check(_native.load().bokt_ep_put(
            flat.data_ptr(), self.a_local * 4, self.ids_ptrs.data_ptr(),
            self.rank * self.a_local * 4, self.world, _native.current_stream(self.device)),
            "bokt_ep_put")
        self._barrier()

    def layout(self):
        """Global routing, per-step layout and this rank's row map."""
        lib = _native.load()
        stream = _native.current_stream(self.device)
        g = self.route_global(self.ids_global)
        _native.check(lib.bokt_ep_plan(
            g.counts.data_ptr(), g.offsets.data_ptr(), self.replicas.data_ptr(), self.experts,
            self.v_rank.data_ptr(), self.V, self.world, self.rank, self.capacity.data_ptr(),
            self.v_plo.data_ptr(), self.v_size.data_ptr(), self.v_lbase.data_ptr(),
            self.loffs.data_ptr(), self.rank_rows.data_ptr(), stream), "bokt_ep_plan")
        _native.check(lib.bokt_ep_rowmap(
            g.perm.data_ptr(), self.ids_global.data_ptr(), g.offsets.data_ptr(),
            g.counts.data_ptr(), self.replicas.data_ptr(), self.vbase.data_ptr(),
            self.v_rank.data_ptr(), self.v_plo.data_ptr(), self.v_lbase.data_ptr(),
            self.a_global, self.experts, self.rank, self.capacity_rows[self.rank],
            self.rowmap.data_ptr(), stream), "bokt_ep_rowmap")

    def dispatch(self, x_local):
        lib = _native.load()
        g = self.route_global
        _native.check(lib.bokt_ep_dispatch(
            x_local.data_ptr(), self.k, x_local.element_size(), self.ids_global.data_ptr(),
            g.inv_perm.data_ptr(), g.offsets.data_ptr(), g.counts.data_ptr(),
            self.replicas.data_ptr(), self.vbase.data_ptr(), self.v_rank.data_ptr(),
            self.v_plo.data_ptr(), self.v_lbase.data_ptr(), self.xpk_ptrs.data_ptr(),
            self.capacity.data_ptr(), self.a_local, self.topk, self.rank, self.experts,
            _native.current_stream(self.device)), "bokt_ep_dispatch")

    def compute_and_combine(self):
        lib = _native.load()
        rows = self.capacity_rows[self.rank]
        if rows == 0:
            return
        _native.check(lib.bokt_moe_grouped_gemm_scatter(
            self.x_packed.data_ptr(), self.w.data_ptr(), self.loffs.data_ptr(), 0, rows,
            self.n_local, self.n, self.k, self.dtype, self.sm, self.rowmap.data_ptr(),
            self.out_ptrs.data_ptr(), self.a_local, self.world, ctypes.byref(self.params),
            _native.current_stream(self.device)), "bokt_moe_grouped_gemm_scatter")

    def barrier_combine(self, gates_local):
        """The step's last barrier with the gate-weighted combine fused into it:
        once every rank's result rows have landed in this rank's ``out``,
        final[t] = sum_j gates[t, j] * out[t * topk + j] (fp32, slot order).
        With ``sync="none"`` (ranks sharing one process) only the combine runs:
        the caller has already ordered the phases."""
        import torch

        g = gates_local.reshape(-1)
        if g.dtype != torch.float32 or g.numel() != self.a_local or not g.is_contiguous():
            raise ValueError("gates_local must be a contiguous fp32 [tokens_per_rank, topk] tensor")
        stream = _native.current_stream(self.device)
        if self.sync == "nccl" and self.world > 1:
            from flashattentionanycard_b200.kernels.moe_routing import combine

            self._barrier()
            combine(self.out, gates_local.reshape(self.tokens_per_rank, self.topk), self.final)
            return self.final
        solo = self.world == 1 or self.sync == "none"
        flags = self._own_flag_ptrs if solo else self.flag_ptrs
        _native.check(_native.load().bokt_ep_barrier_combine(
            flags.data_ptr(), self.epoch.data_ptr(), 1 if solo else self.world,
            0 if solo else self.rank, self.barrier_timeout_ns, self.out.data_ptr(), g.data_ptr(),
            self.final.data_ptr(), self.tokens_per_rank, self.topk, self.n, self.dtype, stream),
            "bokt_ep_barrier_combine")
        return self.final

    def forward(self, x_local, ids_local, gates_local=None, check=False):
        """x_local [tokens_per_rank, K], ids_local [tokens_per_rank, topk] int32 ->

        * without gates: [tokens_per_rank * topk, N] (this rank's output
          buffer, overwritten by the next step), row t*topk + k = x[t] @ W[ids[t, k]];
        * with gates_local [tokens_per_rank, topk] fp32: the MoE layer output in
          token order, [tokens_per_rank, N], row t = sum_k gates[t, k] x[t] @
          W[ids[t, k]] (the combine fused into the step's last barrier).

        ``check=True`` synchronises after the step and raises RuntimeError if a
        kernel recorded a failure (ids out of range, a packed buffer too small
        for this routing, a barrier timeout); without it the step never
        synchronises (graph-capturable) and failures stay in the device status
        word (``_native.device_status``)."""
        self._all_gather_ids(ids_local)
        self.layout()
        self.dispatch(x_local)
        self._barrier()
        self.compute_and_combine()
        if gates_local is None:
            self._barrier()
            result = self.out
        else:
            result = self.barrier_combine(gates_local)
        if check:
            check_device_status(f"expert-parallel step on rank {self.rank}")
        return result
