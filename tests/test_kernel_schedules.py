"""CPU replay of the single-object kernels' row schedules.

The host grid (horner_grid, the open-CTR rows_per_cta split in
confkv_b200/csrc/gpu_aesgcm.cu) cuts an object into tiles; each kernel hands
its tile to the row functions of tiles.cuh, which split the rows into generic
edge rows and the check-free interior loop (replayed in tests/schedules.py).
For every CTA this checks that each row is visited exactly once, that rows
handled by an interior loop satisfy that loop's preconditions (every block
full, inside the object, and -- for open -- not block 0), and that the tiles
of an object cover each block once. The interior loops index memory with no
bounds checks, so this is their bounds proof.
"""

import pytest

from schedules import T, cdiv, ctr_grid, ctr_tile_rows, horner_grid, open_tile_rows, pad_rows, seal_tile_rows

SIZES = [1, 15, 16, 17, 4096, 8191, 8192, 8193, 16 * 512 * 148 - 1, 16 * 512 * 148,
         16 * 512 * 148 + 1, (2 << 20) + 7, 2 << 20, 10 << 20, (32 << 20) + 13, 32 << 20, 1 << 30]


def seal_schedule(n, P, sms):
    iters, grid = horner_grid(n, sms)
    for c in range(grid):
        base = n - (grid - c) * iters * T
        yield c, base, iters, *seal_tile_rows(base, iters, P)


def open_schedule(n, P, sms):
    iters, grid = horner_grid(n, sms)
    for c in range(grid):
        base = n - (grid - c) * iters * T
        yield c, base, iters, *open_tile_rows(base, iters, P)


@pytest.mark.parametrize("sms", [148, 147, 4, 1])
@pytest.mark.parametrize("P", SIZES)
def test_seal_and_open_ghash_rows(P, sms):
    n = cdiv(P, 16)
    for sched in (seal_schedule, open_schedule):
        covered = []
        for c, base, rows, generic, interior in sched(n, P, sms):
            pad = pad_rows(base)
            assert sorted(generic + interior) == list(range(pad, rows)), (sched.__name__, c)
            assert all(base + r * T + T - 1 < 0 for r in range(pad))
            lo_block = 0 if sched is seal_schedule else 1
            for r in interior:
                first, last = base + r * T, base + r * T + T - 1
                assert first >= lo_block and last < P // 16, (sched.__name__, c, r)
            if n < 100000:
                covered += [base + r * T + t for r in range(rows) for t in (0, T - 1) if 0 <= base + r * T + t < n]
        if n < 100000:
            assert len(set(covered)) == len(covered)


@pytest.mark.parametrize("sms", [148, 3, 1])
@pytest.mark.parametrize("P", SIZES)
def test_open_ctr_rows(P, sms):
    n = cdiv(P, 16)
    per, grid = ctr_grid(n, sms)
    rows_total = cdiv(n, T)
    seen = set()
    for c in range(grid):
        row_begin = c * per
        row_end = min(row_begin + per, rows_total)
        generic, interior = ctr_tile_rows(row_begin * T, row_end - row_begin, P)
        assert sorted(generic + interior) == list(range(row_end - row_begin))
        for r in interior:
            row = row_begin + r
            assert row * T >= 1 and (row + 1) * T <= P // 16
        for r in range(row_begin, row_end):
            assert r not in seen
            seen.add(r)
    assert seen == set(range(rows_total))


def test_seal_blocks_each_once_small():
    for P in (1, 4096, 100_003, 16 * 512 * 5 + 3):
        n = cdiv(P, 16)
        for sms in (148, 2):
            blocks = []
            for c, base, rows, generic, interior in seal_schedule(n, P, sms):
                for r in range(rows):
                    blocks += [i for i in range(base + r * T, base + r * T + T) if i >= 0]
            assert sorted(blocks) == list(range(n))


def test_replay_detects_a_wrong_pair_count():
    """The replay catches the class of bug it exists for: an interior loop
    that takes two rows per iteration but counts groups of one row."""
    n_full = (16 * 512 * 7) // 16
    base, rows = 0, 7
    r_hi = min((n_full - base) // T, rows)
    bad_interior = list(range(0, 2 * r_hi))   # would run 2 * 7 rows
    assert any(base + r * T + T - 1 >= n_full for r in bad_interior)
    _, good = seal_tile_rows(base, rows, n_full * 16)
    assert all(base + r * T + T - 1 < n_full for r in good)
