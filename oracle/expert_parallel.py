"""CPU restatement of the expert-parallel MoE dataflow — TEST INFRASTRUCTURE ONLY.

No reference counterpart (the reference is single-GPU).  Given the global
expert ids, a placement (``flashattentionanycard_b200.expert_parallel``) and a
rank, this derives with numpy the orders the device kernels produce
(bokt_ep_keys + stable counting sorts) and runs the whole step for one rank,
with the two exchanges supplied by the caller (real gloo collectives in the
CPU multi-process test).  Arithmetic: fp32 matmul per local virtual expert.
"""

import numpy as np


def rank_orders(ids_flat, placement, topk, tokens_per_rank, rank):
    """Dict of int64 arrays, each a list of packed-row indices p:
    send (rows this rank sends, by destination then p), recv (rows it serves, by
    owner then p), local (rows it serves, by local virtual expert then p), plus
    the global perm, counts of each order and the local expert offsets."""
    world = placement.world
    ids_flat = np.asarray(ids_flat, dtype=np.int64)
    experts = placement.experts
    counts = np.bincount(ids_flat, minlength=experts)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    perm = np.argsort(ids_flat, kind="stable")
    e = ids_flat[perm]
    q = np.arange(perm.size) - offsets[e]
    reps = placement.replicas.astype(np.int64)[e]
    j = (q * reps) // np.maximum(counts[e], 1)
    v = placement.vbase.astype(np.int64)[e] + j
    dest = placement.v_rank.astype(np.int64)[v]
    owner = (perm // topk) // tokens_per_rank
    n_local = len(placement.local[rank])
    key_send = np.where(owner == rank, dest, world)
    key_recv = np.where(dest == rank, owner, world)
    key_local = np.where(dest == rank, placement.v_local.astype(np.int64)[v], n_local)
    out = {"perm": perm, "experts_counts": counts, "offsets": offsets}
    for name, key, buckets in (("send", key_send, world), ("recv", key_recv, world),
                               ("local", key_local, n_local)):
        order = np.argsort(key, kind="stable")
        size = int((key < buckets).sum())
        out[name] = order[:size]
        out[name + "_full"] = order
        out[name + "_counts"] = np.bincount(key, minlength=buckets + 1)[:buckets]
        out[name + "_keys"] = key
    out["local_offsets"] = np.concatenate([[0], np.cumsum(out["local_counts"])])
    return out


def run_rank(x_local, ids_flat, local_weights, placement, topk, tokens_per_rank, rank,
             exchange):
    """One rank's step on the CPU.  ``exchange(send_rows, send_sizes, recv_sizes)``
    returns the received rows (an all-to-all).  Returns the rank's output rows in
    local assignment order, float32 [tokens_per_rank * topk, N]."""
    world = placement.world
    o = rank_orders(ids_flat, placement, topk, tokens_per_rank, rank)
    perm = o["perm"]
    send_sizes = o["send_counts"].astype(np.int64)
    recv_sizes = o["recv_counts"].astype(np.int64)
    x_local = np.asarray(x_local, dtype=np.float32)
    send_x = x_local[perm[o["send"]] // topk - rank * tokens_per_rank]
    recv_x = exchange(send_x, send_sizes, recv_sizes)
    pos_in_recv = np.empty(perm.size, dtype=np.int64)
    pos_in_recv[o["recv"]] = np.arange(o["recv"].size)
    x_packed = recv_x[pos_in_recv[o["local"]]]
    n = local_weights.shape[2]
    y_packed = np.empty((x_packed.shape[0], n), dtype=np.float32)
    lo = o["local_offsets"]
    for lv in range(len(placement.local[rank])):
        s, t = int(lo[lv]), int(lo[lv + 1])
        if t > s:
            y_packed[s:t] = x_packed[s:t] @ np.asarray(local_weights[lv], dtype=np.float32)
    pos_in_local = np.empty(perm.size, dtype=np.int64)
    pos_in_local[o["local"]] = np.arange(o["local"].size)
    y_send = y_packed[pos_in_local[o["recv"]]]
    y_ret = exchange(y_send, recv_sizes, send_sizes)
    inv_perm = np.empty(perm.size, dtype=np.int64)
    inv_perm[perm] = np.arange(perm.size)
    pos_in_send = np.empty(perm.size, dtype=np.int64)
    pos_in_send[o["send"]] = np.arange(o["send"].size)
    a_local = tokens_per_rank * topk
    assignments = np.arange(rank * a_local, (rank + 1) * a_local)
    del world
    return y_ret[pos_in_send[inv_perm[assignments]]]
