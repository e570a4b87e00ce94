"""CPU check of the GEMM's split-tail schedule (the work list every worker of
gemm_sm100_kernel / gemm_sm100_pair_kernel walks, restated from WorkIter and
plan_split in lema_b200/csrc/gemm_sm100.cu): every K-slice of every tile is
computed exactly once; a split tile has exactly two halves on two workers, the
owner (first K-half) and the contributor that publishes the second half into
its own slot; each worker's split half is its last item, so no wait can depend
on a later wait."""
import itertools

import pytest


def plan_split(total_tiles, workers, num_kb, min_kb=8):
    rem = total_tiles % workers
    if rem == 0 or 2 * rem > workers or num_kb < min_kb:
        return total_tiles, 0
    return total_tiles - rem, rem


def work_list(w, W, dp_tiles, split_tiles, num_kb):
    items = [(t, 0, num_kb, "whole", None) for t in range(w, dp_tiles, W)]
    if w < 2 * split_tiles:
        half, h = w & 1, num_kb // 2
        items.append((dp_tiles + w // 2, h if half else 0, num_kb if half else h,
                      "partial" if half else "owner", w + 1))
    return items


CASES = list(itertools.product([1, 5, 31, 32, 34, 40, 74, 100, 256, 300, 768, 1376],
                               [74, 148, 60],
                               [1, 7, 8, 9, 32, 86, 172]))


@pytest.mark.parametrize("tiles,W,num_kb", CASES)
def test_schedule_covers_and_pairs(tiles, W, num_kb):
    dp, split = plan_split(tiles, W, num_kb)
    workers = W if split else min(tiles, W)
    cover = {}
    partial_of, owner_of = {}, {}
    for w in range(workers):
        items = work_list(w, workers, dp, split, num_kb)
        for i, (t, kb0, kb1, role, contrib) in enumerate(items):
            assert 0 <= kb0 < kb1 <= num_kb
            if role != "whole":
                assert i == len(items) - 1  # the split half is the worker's last item
                (partial_of if role == "partial" else owner_of)[w] = t
            if role == "owner":
                assert contrib < workers
            for kb in range(kb0, kb1):
                assert (t, kb) not in cover
                cover[(t, kb)] = w
    assert len(cover) == tiles * num_kb
    assert len(partial_of) == len(owner_of) == split
    for w, t in owner_of.items():
        assert partial_of[w + 1] == t  # the contributor publishes the same tile


def test_plan_default_threshold():
    # default: only tiles of >= 64 K-slices are split (int8 K >= 8192, bf16 K >= 4096)
    assert plan_split(256, 74, 32, min_kb=64) == (256, 0)     # int8 4096^3: whole
    assert plan_split(256, 74, 86, min_kb=64) == (222, 34)    # int8 K = 11008
    assert plan_split(256, 74, 64, min_kb=64) == (222, 34)    # bf16 K = 4096


def test_plan_splits_the_square_4096_gemm():
    # forced (LEMA_GEMM_SPLIT=1): 256 pair tiles of 256 x 256 on 74 pairs,
    # K = 4096 int8 = 32 slices of 128 B
    assert plan_split(256, 74, 32) == (222, 34)
    assert plan_split(768, 74, 32) == (740, 28)
    assert plan_split(1376, 74, 32) == (1376, 0)           # 44 of 74: more than half
    assert plan_split(148 * 3, 148, 32) == (444, 0)        # full waves: no split
    assert plan_split(32, 74, 32) == (0, 32)               # one partial wave, halved
    assert plan_split(256, 74, 4) == (256, 0)              # K too short to halve
