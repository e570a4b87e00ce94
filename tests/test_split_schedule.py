"""CPU check of the GEMM's stream-K schedule: the work list every worker of
gemm_sm100_kernel / gemm_sm100_pair_kernel walks, restated from WorkIter,
plan_schedule, sk_start / sk_worker_of and decode_tile in
lema_b200/csrc/gemm_sm100.cu.

Properties proved over a sweep of tile counts, worker counts and K lengths:
every K-slice of every tile is computed exactly once; every stream-K range is
non-empty; every worker gets the same number of whole tiles after its range; a split tile's owner computes its head (slice 0) and names exactly
the workers that hold the rest of it; a partial item is always its worker's
first item and an owned head its worker's last stream-K item, so an owner only
ever waits on items that wait on nothing; the tile raster is a bijection."""
import itertools

import pytest

K_MIN_UNITS = 8
K_MIN_SLICES = 64
K_FIXUP_SLICES = 4


def plan_schedule(T, W, KB, mode=None):
    """-> (sk_tiles, sk_workers, workers to launch)."""
    whole = min(T, W)
    forced = mode == "1"
    if mode == "0" or T % W == 0 or (not forced and KB < K_MIN_SLICES):
        return 0, 0, whole
    full = T // W
    sk_tiles = T % W
    units = sk_tiles * KB
    S = min(W, units // (1 if forced else K_MIN_UNITS))
    if S < 2:
        return 0, 0, whole
    dp_cost = (full + 1) * KB
    sk_cost = full * KB + -(-units // S) + K_FIXUP_SLICES
    if not forced and sk_cost >= dp_cost:
        return 0, 0, whole
    return sk_tiles, S, (W if full >= 1 else S)


def sk_start(w, units, S):
    return w * units // S


def sk_worker_of(u, units, S):
    return ((u + 1) * S - 1) // units


def work_list(w, W, T, KB, sk_tiles, S):
    units = sk_tiles * KB
    items = []
    if w < S:
        u, u_end = sk_start(w, units, S), sk_start(w + 1, units, S)
        while u < u_end:
            tile = u // KB
            t0, t1 = tile * KB, tile * KB + KB
            stop = min(t1, u_end)
            kb0, kb1 = u - t0, stop - t0
            if kb0 > 0:
                items.append((tile, kb0, kb1, "partial", None))
            elif stop == t1:
                items.append((tile, kb0, kb1, "whole", None))
            else:
                items.append((tile, kb0, kb1, "owner",
                              (sk_worker_of(stop, units, S), sk_worker_of(t1 - 1, units, S))))
            u = stop
    for t in range(sk_tiles + w, T, W):
        items.append((t, 0, KB, "whole", None))
    return items


CASES = list(itertools.product([1, 5, 31, 32, 34, 40, 74, 100, 147, 256, 300, 768, 1376],
                               [74, 148, 60],
                               [1, 7, 8, 9, 32, 86, 172],
                               [None, "1"]))


@pytest.mark.parametrize("T,W,KB,mode", CASES)
def test_schedule_covers_every_slice_once_and_orders_waits(T, W, KB, mode):
    sk_tiles, S, workers = plan_schedule(T, W, KB, mode)
    assert 1 <= workers <= W and S <= workers
    cover = {}
    partial_at = {}   # worker -> (tile, kb0, kb1) of its partial
    owners = {}       # tile -> (owner, c_first, c_last)
    for w in range(workers):
        items = work_list(w, workers, T, KB, sk_tiles, S)
        if w < S:
            assert items and items[0][0] < sk_tiles  # every stream-K range is non-empty
        n_sk = sum(1 for it in items if it[0] < sk_tiles)
        for i, (t, kb0, kb1, role, contrib) in enumerate(items):
            assert 0 <= kb0 < kb1 <= KB
            if role == "partial":
                assert i == 0 and w not in partial_at
                partial_at[w] = (t, kb0, kb1)
            if role == "owner":
                assert i == n_sk - 1 and kb0 == 0
                owners[t] = (w, *contrib)
            for kb in range(kb0, kb1):
                assert (t, kb) not in cover
                cover[(t, kb)] = w
    assert len(cover) == T * KB
    for t, (w, c0, c1) in owners.items():
        assert w < c0 <= c1 < S
        held = sorted(kb for kb in range(KB) if cover[(t, kb)] != w)
        mine = sorted(kb for kb in range(KB) if cover[(t, kb)] == w)
        assert mine == list(range(len(mine)))  # the owner holds the head
        assert {cover[(t, kb)] for kb in held} == set(range(c0, c1 + 1))
        for c in range(c0, c1 + 1):
            assert partial_at[c][0] == t  # each contributor's partial is of this tile
    # every partial is consumed by exactly one owner
    assert sorted(partial_at) == sorted(c for (w, c0, c1) in owners.values()
                                        for c in range(c0, c1 + 1))
    # the whole tiles after the stream-K ranges: the same count for every worker
    dp = [sum(1 for it in work_list(w, workers, T, KB, sk_tiles, S) if it[0] >= sk_tiles)
          for w in range(workers)]
    if sk_tiles:
        assert len(set(dp)) == 1


def test_plan_for_the_training_shapes():
    # int8 M = 4096 on 74 CTA pairs (256 x 256 tiles): K = 4096 -> 32 slices run whole
    assert plan_schedule(256, 74, 32) == (0, 0, 74)         # o, 4096^3
    assert plan_schedule(768, 74, 32) == (0, 0, 74)         # qkv
    assert plan_schedule(256, 74, 86) == (34, 74, 74)       # down, K = 11008: stream-K
    assert plan_schedule(256, 74, 64) == (34, 74, 74)       # bf16 dgrad, K = 4096
    assert plan_schedule(148 * 3, 148, 86) == (0, 0, 148)   # full waves: whole tiles
    assert plan_schedule(256, 74, 86, "0") == (0, 0, 74)    # switched off
    # forced (tests): the K = 4096 shapes too
    assert plan_schedule(256, 74, 32, "1") == (34, 74, 74)
    assert plan_schedule(1376, 74, 32, "1") == (1376 % 74, 74, 74)
    assert plan_schedule(32, 74, 32, "1") == (32, 74, 74)
    assert plan_schedule(4, 148, 4, "1") == (4, 16, 16)
    # a nearly full last wave is not worth the fix-ups
    assert plan_schedule(147, 74, 64) == (0, 0, 74)


def decode(local, m_tiles, n_tiles, raster):
    panel = local // (m_tiles * raster)
    r = local - panel * m_tiles * raster
    width = min(raster, n_tiles - panel * raster)
    mt = r // width
    nt = panel * raster + (r - mt * width)
    return mt, nt


@pytest.mark.parametrize("m_tiles,n_tiles,raster",
                         list(itertools.product([1, 2, 16, 17], [1, 3, 16, 43, 86], [1, 2, 8, 16])))
def test_tile_raster_is_a_bijection(m_tiles, n_tiles, raster):
    raster = max(1, min(raster, n_tiles))
    seen = {decode(t, m_tiles, n_tiles, raster) for t in range(m_tiles * n_tiles)}
    assert seen == {(m, n) for m in range(m_tiles) for n in range(n_tiles)}
    if raster == 1:  # the plain order: row tiles fastest
        assert [decode(t, m_tiles, n_tiles, 1) for t in range(m_tiles)] == \
            [(m, 0) for m in range(m_tiles)]
