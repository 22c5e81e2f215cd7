"""CPU replay of the batched plan and the tile row schedules (batch.cuh,
tiles.cuh): the tile count stays inside the workspace's record area, tiles
partition each object, taller tiles come first in the queue, and every
tile's interior rows meet their loops' preconditions."""

import math

import numpy as np
import pytest

from schedules import (BATCH_EXTRA, SMALL_MAX_BLOCKS, T, batch_plan, cdiv, ctr_tile_rows, open_tile_rows,
                       pad_rows, seal_tile_rows, tile_base)


def _ragged(count, seed, lo=4096, hi=1 << 20):
    rng = np.random.default_rng(seed)
    raw = np.floor(np.exp(rng.uniform(math.log(lo), math.log(hi), size=count))).astype(np.int64)
    return [int(x) + int(rng.integers(0, 16)) for x in raw]


BATCHES = {
    "ragged4096": _ragged(4096, 1),
    "ragged64": _ragged(64, 2),
    "kv_llama8b_x32": [32 << 20] * 32,
    "one_huge": [(1 << 30) + 7],
    "huge_and_tiny": [1 << 30, 1, 0, 17, 4096] * 3,
    "zeros": [0] * 100,
    "tiny_many": list(range(0, 20000, 7)),
    "max_blocks": [16 * 0xFFFFFFFE, 5],
}


@pytest.mark.parametrize("name", sorted(BATCHES))
@pytest.mark.parametrize("sms", [148, 132, 1, 300])
def test_plan_bound_order_and_partition(name, sms):
    lens = BATCHES[name]
    jstar, plan, queue = batch_plan(lens, sms)
    assert len(queue) <= len(lens) + BATCH_EXTRA
    # taller tiles first
    js = [plan[i][0] for i, _ in queue]
    assert all((a.bit_length() >= b.bit_length()) for a, b in zip(js, js[1:]))
    assert len(set(queue)) == len(queue)
    for i, P in enumerate(lens):
        n = cdiv(P, 16)
        if n <= SMALL_MAX_BLOCKS:
            assert plan[i] is None and all(q[0] != i for q in queue)   # one warp, no tiles
            continue
        J, G = plan[i]
        assert 1 <= J <= jstar and G >= 1
        assert sum(1 for q in queue if q[0] == i) == G if len(lens) < 200 else True
        # tiles cover [0, n) exactly once; only tile 0 may start below 0
        starts = [tile_base(n, J, G, c) for c in range(G)]
        assert starts[-1] + J * T == n
        assert all(b >= 0 for b in starts[1:])
        assert starts[0] > -J * T or n == 0
        # a one-tile object uses exactly its rows (no wasted rows)
        if G == 1:
            assert J == max(1, cdiv(n, T))


def test_plan_tile_height():
    # 32 x 32 MiB: eight equal waves of 111-row tiles (37 per object)
    jstar, plan, queue = batch_plan([32 << 20] * 32, 148)
    assert jstar == 111 and len(queue) == 32 * 37 == 8 * 148
    # one 32 MiB object: one wave
    jstar, plan, queue = batch_plan([32 << 20], 148)
    assert len(queue) <= 148 and jstar == 28
    # 64 x 1 MiB: every object in two tiles -> 128 tiles, one wave
    jstar, plan, queue = batch_plan([1 << 20] * 64, 148)
    assert jstar == 64 and len(queue) == 128
    # 64 x 2 MiB kv_small objects: two tiles each
    jstar, plan, queue = batch_plan([2 << 20] * 64, 148)
    assert jstar == 128 and len(queue) == 128
    # all invalid / empty
    assert batch_plan([5, 6], 148, valid=[False, False])[0] == 1


def test_plan_skips_invalid():
    lens = [100, 200, 300]
    jstar, plan, queue = batch_plan(lens, 148, valid=[True, False, True])
    assert plan[1] is None and all(q[0] != 1 for q in queue)


def _check_tile(base, rows, P, lo_block, sched, hi_margin=0):
    generic, interior = sched(base, rows, P)
    pad = pad_rows(base)
    assert sorted(generic + interior) == list(range(pad, rows))
    # skipped rows hold no block of the object
    assert all(base + r * T + T - 1 < 0 for r in range(pad))
    n_full = P // 16
    for r in interior:
        assert base + r * T >= lo_block and base + r * T + T - 1 < n_full - hi_margin, (base, rows, P, r)


SIZES = [0, 1, 15, 16, 17, 4095, 4096, 8191, 8192, 8193, 16 * 512 * 3 + 5, 16 * 512 * 80 - 1, (1 << 20) + 15,
         (32 << 20) + 13, 1 << 30]


@pytest.mark.parametrize("P", SIZES)
@pytest.mark.parametrize("J", [1, 2, 3, 7, 80, 222])
def test_tile_rows_every_tile(P, J):
    n = cdiv(P, 16)
    J = max(1, min(J, cdiv(n, T) if n else 1))
    G = max(1, cdiv(n, J * T))
    tiles = range(G) if G <= 64 else list(range(3)) + list(range(G - 3, G))
    for c in tiles:
        base = tile_base(n, J, G, c)
        _check_tile(base, J, P, 0, seal_tile_rows)
        # misaligned plaintext: both aligned chunks of every interior block
        # lie inside the object
        _check_tile(base, J, P, 1, lambda b, r, p: seal_tile_rows(b, r, p, pt_aligned=False), hi_margin=1)
        _check_tile(base, J, P, 1, open_tile_rows)
        _check_tile(base, J, P, 1, ctr_tile_rows)
