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


def _written_partials(ntiles, split, nkb, launched):
    """(tile, worker, which) of every partial the GEMM epilogue stores in the
    separate-reduction mode: a segment that does not cover its whole tile goes
    to slot 0 when it is the first of its worker's run, else slot 1."""
    out = {}
    index = {}
    for w, t, k0, k1, _, _ in _native.splitk_schedule(ntiles, split, nkb, launched):
        i = index.get(w, 0)
        index[w] = i + 1
        if k0 > 0 or k1 < nkb:
            key = (w, 1 if i > 0 else 0)
            assert key not in out, "two partials written into one slot"
            out[key] = (t, k0, k1)
    return out


@pytest.mark.parametrize("ntiles", [1, 2, 3, 16, 64, 120, 1024])
def test_reduce_sources_match_written_partials(ntiles):
    """Every partial the reduction reads was written for that tile, every
    written partial is read exactly once, and per tile the reads run in worker
    order over k-blocks 0 .. nkb without gaps."""
    checked = 0
    for split, nkb, launched in itertools.product((4, 5, 16, 64, 128), (4, 16, 65, 1024),
                                                  (1, 5, 74, 148)):
        written = _written_partials(ntiles, split, nkb, launched)
        sources = _native.splitk_reduce_sources(ntiles, split, nkb, launched)
        seen = set()
        by_tile = {}
        for t, w, which in sources:
            assert which in (0, 1)
            assert (w, which) in written, "reduction reads a slot nothing wrote"
            assert written[(w, which)][0] == t, "slot holds another tile's partial"
            assert (w, which) not in seen
            seen.add((w, which))
            by_tile.setdefault(t, []).append(written[(w, which)])
        assert seen == set(written), "a written partial is never read"
        for t, parts in by_tile.items():
            assert len(parts) >= 2
            assert parts[0][1] == 0 and parts[-1][2] == nkb
            assert all(a[2] == b[1] for a, b in zip(parts, parts[1:]))
        checked += len(sources)
    assert checked > 0


def test_reduce_tall_k_pairs():
    """256 x 256 x 65536 on 74 pairs with 64 slices: the single tile is summed
    from the partials of all 64 workers."""
    sources = _native.splitk_reduce_sources(1, 64, 1024, 74)
    assert [w for _, w, _ in sources] == list(range(64))
    assert all(which == 0 for *_, which in sources)
