"""CPU replay of the seal / open kernels' row schedules.

Mirrors, line for line, the host grid computation (horner_grid, the open-CTR
rows_per_cta split in confkv_b200/csrc/gpu_aesgcm.cu) and each kernel's split
of its rows into generic edge rows and the check-free interior loop. For every
CTA it checks that each row is visited exactly once, that rows handled by the
interior loop satisfy that loop's preconditions (every block full, inside the
object, and -- for open -- not block 0), and that the interior loop's
prefetches stay inside the interior range. The kernels index memory with no
bounds checks in the interior loop, so this is the bounds proof for it.
"""

import pytest

T_ROW = 512      # kHornerThreads
T_CTR = 512      # kCtrThreads
SEAL_PAIR = 2    # rows per interior iteration in seal_kernel
OPEN_R = 2       # kOpenChains: rows per interior iteration in open_ghash_kernel
CTR_PAIR = 2


def horner_grid(n, sms):
    per_wave = sms * T_ROW
    j = max(1, -(-n // per_wave))
    span = j * T_ROW
    return j, -(-n // span)


def seal_schedule(n, P, sms):
    iters, grid = horner_grid(n, sms)
    span = iters * T_ROW
    n_full = P // 16
    for c in range(grid):
        base = n - (grid - c) * span
        rows = iters
        r_lo = 0 if base >= 0 else (-base + T_ROW - 1) // T_ROW
        r_hi = min((n_full - base) // T_ROW, rows)
        r_a = min((r_lo + SEAL_PAIR - 1) // SEAL_PAIR * SEAL_PAIR, r_hi)
        ngroups = (r_hi - r_a) // SEAL_PAIR if r_hi > r_a else 0
        generic = list(range(0, r_a)) + list(range(r_a + SEAL_PAIR * ngroups, rows))
        interior = list(range(r_a, r_a + SEAL_PAIR * ngroups))
        yield c, base, rows, generic, interior, n_full


def open_schedule(n, P, sms):
    iters, grid = horner_grid(n, sms)
    span = iters * T_ROW
    n_full = P // 16
    for c in range(grid):
        base = n - (grid - c) * span
        rows = iters
        r_lo = 0 if base >= 1 else (1 - base + T_ROW - 1) // T_ROW
        r_hi = min((n_full - base) // T_ROW, rows)
        r_a = min((r_lo + OPEN_R - 1) // OPEN_R * OPEN_R, r_hi)
        ngroups = (r_hi - r_a) // OPEN_R if r_hi > r_a else 0
        generic = list(range(0, r_a)) + list(range(r_a + OPEN_R * ngroups, rows))
        interior = list(range(r_a, r_a + OPEN_R * ngroups))
        yield c, base, rows, generic, interior, n_full


def ctr_schedule(n, P, sms):
    rows_total = -(-n // T_CTR)
    per = -(-rows_total // sms)
    grid = -(-rows_total // per)
    n_full = P // 16
    for c in range(grid):
        row_begin = c * per
        row_end = min(row_begin + per, rows_total)
        r_lo = max(row_begin, 1)
        r_hi = min(n_full // T_CTR, row_end)
        if r_lo > r_hi:
            r_lo = r_hi = row_end
        npair = (r_hi - r_lo) // CTR_PAIR
        generic = list(range(row_begin, r_lo)) + list(range(r_lo + CTR_PAIR * npair, row_end))
        interior = list(range(r_lo, r_lo + CTR_PAIR * npair))
        yield c, row_begin, row_end, generic, interior, n_full


SIZES = [1, 15, 16, 17, 4096, 8191, 8192, 8193, 16 * 512 * 148 - 1, 16 * 512 * 148,
         16 * 512 * 148 + 1, (2 << 20) + 7, 2 << 20, 10 << 20, (32 << 20) + 13, 32 << 20, 1 << 30]


@pytest.mark.parametrize("sms", [148, 147, 4, 1])
@pytest.mark.parametrize("P", SIZES)
def test_seal_and_open_ghash_rows(P, sms):
    n = -(-P // 16)
    for sched in (seal_schedule, open_schedule):
        covered = []
        for c, base, rows, generic, interior, n_full in sched(n, P, sms):
            assert sorted(generic + interior) == list(range(rows)), (sched.__name__, c)
            lo_block = 0 if sched is seal_schedule else 1
            for r in interior:
                first, last = base + r * T_ROW, base + r * T_ROW + T_ROW - 1
                assert first >= lo_block and last < n_full, (sched.__name__, c, r)
            covered += [base + r * T_ROW + t for r in range(rows) for t in (0, T_ROW - 1)
                        if 0 <= base + r * T_ROW + t < n] if n < 100000 else []
            # interior loop prefetches the next group only while one remains
            if interior:
                assert interior[-1] < rows
        if n < 100000:
            assert len(set(covered)) == len(covered)


@pytest.mark.parametrize("sms", [148, 3, 1])
@pytest.mark.parametrize("P", SIZES)
def test_open_ctr_rows(P, sms):
    n = -(-P // 16)
    seen = set()
    for c, row_begin, row_end, generic, interior, n_full in ctr_schedule(n, P, sms):
        assert sorted(generic + interior) == list(range(row_begin, row_end))
        for r in interior:
            assert r >= 1 and (r + 1) * T_CTR <= n_full
        for r in range(row_begin, row_end):
            assert r not in seen
            seen.add(r)
    assert seen == set(range(-(-n // T_CTR)))


def test_seal_blocks_each_once_small():
    for P in (1, 4096, 100_003, 16 * 512 * 5 + 3):
        n = -(-P // 16)
        for sms in (148, 2):
            blocks = []
            for c, base, rows, generic, interior, n_full in seal_schedule(n, P, sms):
                for r in range(rows):
                    blocks += [i for i in range(base + r * T_ROW, base + r * T_ROW + T_ROW) if i >= 0]
            assert sorted(blocks) == list(range(n))
