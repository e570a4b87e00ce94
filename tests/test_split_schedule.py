"""CPU check of the GEMM's split-tail schedule (the work list every worker of
gemm_sm100_kernel / gemm_sm100_pair_kernel walks, restated from WorkIter and
plan_split in lema_b200/csrc/gemm_sm100.cu): every K-slice of every tile is
computed exactly once; each worker publishes at most one partial (its slot is
its own) and does so in its first tail segment; an owner's segment is its last
and its contributor list is exactly the set of workers that publish a partial
of its tile; so no wait can depend on a later wait."""
import itertools

import pytest


def plan_split(total_tiles, workers, num_kb):
    rem = total_tiles % workers
    if rem == 0 or rem * 20 > workers * 17:
        return total_tiles, 0
    units = rem * num_kb
    if units < 4 * workers or units > 2**31 - 1:
        return total_tiles, 0
    return total_tiles - rem, units


def work_list(w, W, dp_tiles, tail_units, num_kb):
    items = [(t, 0, num_kb, "whole", []) for t in range(w, dp_tiles, W)]
    begin = lambda q: q * tail_units // W
    u, e = begin(w), begin(w + 1)
    while u < e:
        tl = u // num_kb
        t0, t1 = tl * num_kb, (tl + 1) * num_kb
        end = min(e, t1)
        kb0, kb1 = u - t0, end - t0
        contrib = []
        if kb0 > 0:
            role = "partial"
        elif kb1 < num_kb:
            role = "owner"
            for q in range(w + 1, W):
                bq = begin(q)
                if bq >= t1:
                    break
                if bq > t0 and begin(q + 1) > bq:
                    contrib.append(q)
        else:
            role = "whole"
        items.append((dp_tiles + tl, kb0, kb1, role, contrib))
        u = end
    return items


CASES = list(itertools.product([1, 5, 31, 32, 34, 40, 74, 100, 256, 300, 768, 1376],
                               [74, 148, 60],
                               [1, 2, 3, 4, 8, 32, 86, 172]))


@pytest.mark.parametrize("tiles,W,num_kb", CASES)
def test_schedule_covers_and_orders(tiles, W, num_kb):
    dp, units = plan_split(tiles, W, num_kb)
    workers = W if units else min(tiles, W)
    cover = {}
    partial_of = {}
    owners = {}
    for w in range(workers):
        items = work_list(w, workers, dp, units, num_kb)
        parts = [i for i, it in enumerate(items) if it[3] == "partial"]
        assert len(parts) <= 1
        if parts:
            assert parts[0] == sum(1 for it in items if it[0] < dp)  # first tail segment
            partial_of[w] = items[parts[0]][0]
        own = [i for i, it in enumerate(items) if it[3] == "owner"]
        assert len(own) <= 1
        if own:
            assert own[0] == len(items) - 1  # last segment
            owners[items[own[0]][0]] = (w, items[own[0]][4])
        for t, kb0, kb1, role, _ in items:
            assert 0 <= kb0 < kb1 <= num_kb
            for kb in range(kb0, kb1):
                assert (t, kb) not in cover
                cover[(t, kb)] = w
    assert len(cover) == tiles * num_kb
    # contributors of each owned tile == the workers publishing a partial of it
    for t, (w, contrib) in owners.items():
        assert sorted(q for q, pt in partial_of.items() if pt == t) == contrib
        assert all(q > w for q in contrib)
    # every partial has an owner that reads it
    for q, t in partial_of.items():
        assert t in owners and q in owners[t][1]


def test_plan_splits_the_square_4096_gemm():
    # 256 pair tiles of 256 x 256 on 74 pairs, K = 4096 int8 = 32 slices of 128 B
    dp, units = plan_split(256, 74, 32)
    assert dp == 222 and units == 34 * 32
    assert plan_split(1376, 74, 32) == (1332, 44 * 32)
    assert plan_split(148 * 3, 148, 32) == (444, 0)        # full waves: no split
    assert plan_split(70, 74, 32) == (70, 0)               # last wave 95 % full
