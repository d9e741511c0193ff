"""The split-K schedule the kernels run, checked on the host (no GPU): the
library's own host copy of the device arithmetic (bokt_splitk_schedule)."""

import itertools

import pytest

from flashattentionanycard_b200 import _native


def _check(ntiles, split, nkb, launched):
    segs = _native.splitk_schedule(ntiles, split, nkb, launched)
    eff = min(split, nkb)
    cover = set()
    by_worker = {}
    for w, t, k0, k1, first, count in segs:
        assert 0 <= t < ntiles and 0 <= k0 < k1 <= nkb
        by_worker.setdefault(w, []).append((t, k0, k1))
        for kb in range(k0, k1):
            assert (t, kb) not in cover, "k-block computed twice"
            cover.add((t, kb))
    assert len(cover) == ntiles * nkb, "k-block never computed"
    for t in range(ntiles):
        owners = [s for s in segs if s[1] == t and s[2] == 0]
        assert len(owners) == 1, "a tile needs exactly one owner"
        w, _, _, k1, first, count = owners[0]
        others = sorted(s[0] for s in segs if s[1] == t and s[2] > 0)
        if eff == 1:
            assert not others
        # The owner adds exactly the partials of the tile's other segments,
        # which belong to the workers right after it.
        assert others == (list(range(first, first + count)) if k1 < nkb else [])
    for w, run in by_worker.items():
        # A non-owner segment is the first of its worker's run (it never waits).
        assert all(k0 == 0 for _, k0, _ in run[1:])
    if eff > 1:
        # Balanced: runs differ by at most one unit of k-blocks.
        sizes = [sum(k1 - k0 for _, k0, k1 in run) for run in by_worker.values()]
        unit = -(-nkb // eff)
        assert max(sizes) - min(sizes) <= 2 * unit
    return len(segs)


@pytest.mark.parametrize("ntiles", [1, 3, 16, 64, 120, 1024])
def test_schedule_invariants(ntiles):
    n = 0
    for split, nkb, launched in itertools.product((1, 2, 3, 8, 16, 32), (1, 2, 5, 16, 32, 65),
                                                  (1, 5, 74, 148)):
        n += _check(ntiles, split, nkb, launched)
    assert n > 0


def test_stream_k_2048_pairs():
    """2048^3 on 74 CTA pairs with 8 slices of 4 k-blocks: every pair runs 24 or
    28 k-blocks instead of 32 (one partial wave of 64 whole tiles)."""
    segs = _native.splitk_schedule(64, 8, 32, 74)
    per = {}
    for w, t, k0, k1, _, _ in segs:
        per[w] = per.get(w, 0) + (k1 - k0)
    assert len(per) == 74 and max(per.values()) == 28 and min(per.values()) == 24
    assert segs[0] == (0, 0, 0, 24, 1, 1)
