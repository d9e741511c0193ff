"""MoE routing oracle: histogram, offsets, stable permutation, combine indices.

Test infrastructure only (see ``oracle/__init__.py``).  The reference builds
offsets as a host prefix sum of per-expert token counts
(``bo_kernel_tuner/tuner/worker.py:83-86``); the permutation and its inverse
have no reference counterpart and are defined here as a stable counting sort:
assignment i (flattened token-major, ``i = token * topk + slot``) lands at
packed row ``offsets[e] + #{j < i : id[j] == e}``.
"""

import numpy as np


def expert_counts(ids, experts):
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    if ids.size and (ids.min() < 0 or ids.max() >= experts):
        raise ValueError("expert id out of range")
    counts = np.zeros(experts, dtype=np.int64)
    for e in ids:  # explicit histogram (cross-checked against np.bincount in tests)
        counts[e] += 1
    return counts.astype(np.int32)


def expert_offsets(counts):
    """Exclusive prefix sum with the total appended (worker.py:83-86)."""
    out = [0]
    for c in np.asarray(counts).tolist():
        out.append(out[-1] + int(c))
    return np.asarray(out, dtype=np.int64)


def stable_permutation(ids, experts):
    """perm[row] = assignment index; rows grouped by expert, stable inside an expert."""
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    offsets = expert_offsets(expert_counts(ids, experts))
    cursor = offsets[:-1].copy()
    perm = np.empty(ids.size, dtype=np.int64)
    for i, e in enumerate(ids.tolist()):
        perm[cursor[e]] = i
        cursor[e] += 1
    return perm.astype(np.int32)


def inverse_permutation(perm):
    perm = np.asarray(perm, dtype=np.int64)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size, dtype=np.int64)
    return inv.astype(np.int32)


def route(ids, experts):
    """(counts int32[E], offsets int64[E+1], perm int32[A], inv_perm int32[A])."""
    counts = expert_counts(ids, experts)
    perm = stable_permutation(ids, experts)
    return counts, expert_offsets(counts), perm, inverse_permutation(perm)



def topk_gate(logits, k, renormalize=True):
    """(ids int32 [T, k], gates float32 [T, k]): the k largest logits per row
    (ties: lower expert index first) and their softmax probabilities, computed
    in float64 and optionally renormalised over the picked experts."""
    logits = np.asarray(logits, dtype=np.float64)
    t, e = logits.shape
    order = np.lexsort((np.broadcast_to(np.arange(e), (t, e)), -logits), axis=-1)
    ids = order[:, :k]
    z = logits - logits.max(axis=1, keepdims=True)
    p = np.exp(z) / np.exp(z).sum(axis=1, keepdims=True)
    gates = np.take_along_axis(p, ids, axis=1)
    if renormalize:
        gates = gates / gates.sum(axis=1, keepdims=True)
    return ids.astype(np.int32), gates.astype(np.float32)


def combine(y, gates, rows=None):
    """out[t] = sum_j gates[t, j] * y[row(t, j)] in float32."""
    y = np.asarray(y, dtype=np.float32)
    gates = np.asarray(gates, dtype=np.float32)
    t, k = gates.shape
    idx = np.arange(t * k) if rows is None else np.asarray(rows, dtype=np.int64)
    picked = y[idx].reshape(t, k, -1)
    return np.einsum("tk,tkn->tn", gates, picked).astype(np.float32)
