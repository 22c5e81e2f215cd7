"""CPU replay of the batched plan and the row schedules (batch.cuh,
tiles.cuh): the chunks cut the row space into near-equal pieces that fit the
workspace, walking every chunk's segments covers each tile object's rows
exactly once with the segment count its slot expects, and every segment's
interior rows meet their loops' preconditions."""

import math

import numpy as np
import pytest

from schedules import (MAX_CHUNKS, SEGMENT_COST_ROWS, SMALL_MAX_BLOCKS, T, cdiv, chunk_plan, chunk_segments, ctr_tile_rows,
                       mid_routed, OPEN_BATCH_R, open_tile_rows, pad_rows, seal_tile_rows, segment_base, tile_base, tile_rows)


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
    "just_above_small": [SMALL_MAX_BLOCKS * 16 + 1] * 7,
    # mid objects (16-32 KiB): few stay tile objects, many take one warp each
    "mid_few": [32768, 24576, 16385, 32767, 4096] * 40,
    "mid_many": [32768, 20480, 16400, 2048] * 400,
}


def _walk(plan):
    """All chunks' segments in chunk order."""
    return [seg for c in range(plan["M"]) for seg in chunk_segments(plan, c)]


@pytest.mark.parametrize("name", sorted(BATCHES))
@pytest.mark.parametrize("sms", [148, 132, 1, 300])
@pytest.mark.parametrize("mixed", [False, True])
@pytest.mark.parametrize("open_", [False, True])
def test_chunks_cover_every_row_once(name, sms, mixed, open_):
    lens = BATCHES[name]
    classes = [(7 * i) % 10 for i in range(len(lens))] if mixed else None
    plan = chunk_plan(lens, sms, classes=classes, open_=open_)
    R, M = plan["R"], plan["M"]
    routed = plan["mid_routed"]
    assert routed == mid_routed(lens, min(sms, 256), open_=open_)
    assert R == sum(tile_rows(P, True, routed) for P in lens)
    assert M <= MAX_CHUNKS and M <= R and (M > 0) == (R > 0)
    # chunks are non-empty and of near-equal cost: rows plus a charge per
    # segment, within two charges and one row of each other
    o = SEGMENT_COST_ROWS
    starts = plan["chunk_start"]
    assert all(a < b for a, b in zip(starts, starts[1:]))
    costs = [sum(r1 - r0 for _, _, r0, r1 in chunk_segments(plan, c)) + o * len(chunk_segments(plan, c))
             for c in range(M)]
    if M and (R + o * len(plan["objs"])) // M >= 2 * (o + 1):
        assert max(costs) - min(costs) <= 2 * o + 1
    segs = _walk(plan)
    covered = {}
    count = {}
    if mixed:
        # grouped by class: the class changes at most 9 times along the row space
        cls = [classes[item] for item, _, _, _ in segs]
        assert sum(a != b for a, b in zip(cls, cls[1:])) <= 9
    for item, rows, r0, r1 in segs:
        assert 0 <= r0 < r1 <= rows == tile_rows(lens[item], True, routed)
        covered.setdefault(item, []).append((r0, r1))
        count[item] = count.get(item, 0) + 1
    for i, P in enumerate(lens):
        rows = tile_rows(P, True, routed)
        if rows == 0:
            assert i not in covered and plan["segments"][i] == 0   # small or empty: one warp, no segments
            continue
        spans = covered[i]
        # in order, contiguous, covering [0, rows)
        assert spans[0][0] == 0 and spans[-1][1] == rows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert count[i] == plan["segments"][i]


def test_chunk_counts():
    # 32 x 32 MiB (few objects): one chunk per SM of 885-886 rows
    plan = chunk_plan([32 << 20] * 32, 148)
    assert plan["R"] == 32 * 4096 and plan["M"] == 148
    # 4096 ragged objects (many): four chunks per SM
    assert chunk_plan(BATCHES["ragged4096"], 148)["M"] == 4 * 148
    # 64 x 2 MiB: one chunk per SM (110-111 rows), objects cut across chunks
    plan = chunk_plan([2 << 20] * 64, 148)
    assert plan["M"] == 148 and set(plan["segments"]) == {3, 4}
    # one 32 MiB object: 148 chunks of 27-28 rows, 148 segments
    plan = chunk_plan([32 << 20], 148)
    assert plan["M"] == 148 and plan["segments"][0] == 148
    # fewer rows than SMs: one row per chunk
    plan = chunk_plan([20000] * 10, 148)   # 3 rows each
    assert plan["R"] == 30 and plan["M"] == 30
    # nothing to tile
    assert chunk_plan([5, 6], 148, valid=[False, False])["M"] == 0
    assert chunk_plan([], 148)["M"] == 0


def test_mid_objects_take_the_warp_path_only_in_number():
    sms = 148
    # 2048 objects of 32 KiB: 13.8 per SM, one warp each
    plan = chunk_plan([32768] * 2048, sms)
    assert plan["mid_routed"] and plan["R"] == 0 and plan["M"] == 0
    # crossovers of 32 KiB objects: seal from 26 * 2048 / (9 * 512) = 11.6
    # objects per SM, open from 19 * 2048 / (9 * 512) = 8.4
    assert not mid_routed([32768] * 1710, sms) and mid_routed([32768] * 1711, sms)
    assert not mid_routed([32768] * 1249, sms, open_=True) and mid_routed([32768] * 1250, sms, open_=True)
    plan = chunk_plan([32768] * 1480, sms)
    assert not plan["mid_routed"] and plan["R"] == 4 * 1480
    assert chunk_plan([32768] * 1480, sms, open_=True)["mid_routed"]
    # 20 KiB objects (3 rows as tiles, 40 as a warp): seal from 8.1 per SM
    assert not mid_routed([20480] * 1202, sms) and mid_routed([20480] * 1203, sms)
    # small objects count toward N; larger objects stay tiles
    lens = [32768] * 10 + [4096] * 1702 + [1 << 20] * 3
    plan = chunk_plan(lens, sms)
    assert plan["mid_routed"] and plan["R"] == 3 * 128
    # without mid objects there is nothing to route
    assert not chunk_plan([4096] * 5000, sms)["mid_routed"]
    # invalid descriptors do not count; a mixed batch can route open only
    assert not mid_routed([32768] * 1711, sms, valid=[True] * 1710 + [False])
    mixed = [32768, 20480, 16400, 2048] * 400
    assert not mid_routed(mixed, sms) and mid_routed(mixed, sms, open_=True)
    assert tile_rows(32768) == 4 and tile_rows(32768, True, True) == 0
    assert tile_rows(32784, True, True) == 5   # 2049 blocks: above the warp path


def test_plan_skips_invalid():
    lens = [1 << 20, 2 << 20, 3 << 20]
    plan = chunk_plan(lens, 148, valid=[True, False, True])
    assert plan["segments"][1] == 0 and all(seg[0] != 1 for seg in _walk(plan))


@pytest.mark.parametrize("name", ["ragged64", "huge_and_tiny", "kv_llama8b_x32", "just_above_small", "max_blocks"])
def test_segment_rows_meet_loop_preconditions(name):
    lens = BATCHES[name]
    plan = chunk_plan(lens, 148)
    segs = _walk(plan)
    if len(segs) > 400:
        segs = segs[:200] + segs[-200:]
    for item, rows, r0, r1 in segs:
        P = lens[item]
        base = segment_base(P, rows, r0)
        J = r1 - r0
        _check_tile(base, J, P, 0, seal_tile_rows)
        _check_tile(base, J, P, 1, lambda b, r, p: seal_tile_rows(b, r, p, pt_aligned=False), hi_margin=1)
        _check_tile(base, J, P, 1, lambda b, r, p: open_tile_rows(b, r, p, R=OPEN_BATCH_R))
        _check_tile(base, J, P, 1, ctr_tile_rows)


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
        _check_tile(base, J, P, 1, lambda b, r, p: open_tile_rows(b, r, p, R=OPEN_BATCH_R))
        _check_tile(base, J, P, 1, ctr_tile_rows)
