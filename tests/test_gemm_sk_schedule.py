"""Host model of the stream-K GEMM's schedule (csrc/gemm_sk.cu: range_lo,
SegIter, the owner / contributor rule), run over the plans the library makes
for the Qwen3 decode projections (CPU; no GPU needed):

* the pairs' ranges partition the (tile, K-step) iterations, none empty;
* every tile is covered by pieces in K order whose union is its K range;
* a cut tile's first piece (its owner) is the LAST segment of its pair and
  every later piece (a contributor) is the FIRST segment of a later pair, so
  a pair contributes at most once (one partial slot and one flag per pair);
* the owner's contributor list (pairs after it whose range starts inside its
  tile) is exactly the tile's later pieces, so every raised flag is consumed
  and reset by exactly one owner in the same launch;
* owners only wait for first segments, which wait for nothing: with every
  pair resident (one wave) the hand-off cannot deadlock.
"""
import pytest


def range_lo(p, iters, pairs):
    return p * iters // pairs  # 32-bit on the device; the host keeps pairs * iters < 2^32


def segments(lo, hi, kb):
    it = lo
    while it < hi:
        tile = it // kb
        k0 = it - tile * kb
        k1 = min(kb, k0 + (hi - it))
        yield tile, k0, k1
        it += k1 - k0


def check_schedule(tiles, kb, pairs, ranges=None):
    iters = tiles * kb
    assert pairs * iters < 2 ** 32
    if ranges is None:
        ranges = [(range_lo(p, iters, pairs), range_lo(p + 1, iters, pairs)) for p in range(pairs)]
    pieces = {}          # tile -> [(k0, k1, pair, segment index, segments of the pair)]
    for p in range(pairs):
        lo, hi = ranges[p]
        assert hi > lo, "empty range"
        segs = list(segments(lo, hi, kb))
        contributors = [s for s in segs if s[1] > 0]
        assert len(contributors) <= 1, "a pair contributes at most once"
        if contributors:
            assert segs[0] == contributors[0], "a contributor is its pair's first segment"
        for j, (t, k0, k1) in enumerate(segs):
            pieces.setdefault(t, []).append((k0, k1, p, j, len(segs)))
    assert sorted(pieces) == list(range(tiles))
    flags_raised, flags_consumed = set(), []
    for t, ps in pieces.items():
        ps.sort()
        assert ps[0][0] == 0 and ps[-1][1] == kb
        for a, b in zip(ps, ps[1:]):
            assert a[1] == b[0], "pieces of a tile are contiguous in K"
        if len(ps) == 1:
            continue
        owner = ps[0]
        assert owner[3] == owner[4] - 1, "the owner piece is the last segment of its pair"
        # the owner's list: pairs after it whose range starts inside the tile
        tile_end = (t + 1) * kb
        c_last = owner[2]
        while c_last + 1 < pairs and ranges[c_last + 1][0] < tile_end:
            c_last += 1
        listed = list(range(owner[2] + 1, c_last + 1))
        assert listed == [q[2] for q in ps[1:]], (t, listed, ps)
        for q in ps[1:]:
            assert q[3] == 0, "a contributor piece is the first segment of its pair"
            flags_raised.add(q[2])
        flags_consumed += listed
    assert sorted(flags_consumed) == sorted(flags_raised), "every flag is consumed once"
    return len(flags_raised)


SHAPES = [(M, N, K, g) for M in (1, 16, 64, 256) for (N, K, g) in (
    (6144, 4096, False), (4096, 4096, False), (12288, 4096, True), (4096, 12288, False), (151936, 4096, False),
    (768, 4096, False), (4096, 512, False), (1536, 4096, True), (4096, 1536, False), (18992, 4096, False))]


@pytest.fixture(scope="module")
def K():
    from kavor_b200 import _kernels, _lib, build

    build.build()
    _lib.load()
    return _kernels


@pytest.mark.parametrize("M,N,Kd,gated", SHAPES)
def test_planned_schedule_hands_off_every_partial_once(K, M, N, Kd, gated):
    p = K.gemm_sk_plan(M, N, Kd, gated)
    check_schedule(p["tiles"], p["kb"], p["pairs"])


@pytest.mark.parametrize("tiles,kb", [(1, 1), (1, 64), (3, 32), (24, 32), (16, 4), (594, 22), (7, 5)])
def test_every_pair_count_hands_off_every_partial_once(tiles, kb):
    for pairs in range(1, min(128, tiles * kb) + 1):
        check_schedule(tiles, kb, pairs)


def test_the_model_finds_a_broken_rule():
    """The checks are not vacuous: dealing the same ranges to the pairs in
    reverse order (pair 0 the last range, ...) breaks the owner's rule for
    finding its contributors (the pairs after it whose range starts inside
    its tile): the listed pairs are no longer the tile's later pieces, and the
    model rejects it; so does an empty range."""
    tiles, kb, pairs = 24, 32, 70
    iters = tiles * kb
    fwd = [(range_lo(p, iters, pairs), range_lo(p + 1, iters, pairs)) for p in range(pairs)]
    assert check_schedule(tiles, kb, pairs, fwd) > 0
    with pytest.raises(AssertionError):
        check_schedule(tiles, kb, pairs, fwd[::-1])
    with pytest.raises(AssertionError):
        check_schedule(2, 8, 20)  # more pairs than iterations: an empty range
