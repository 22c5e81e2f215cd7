"""CPU replays of the kernels' index arithmetic (test infrastructure).

Each function restates, line for line, one piece of confkv_b200/csrc:
  tile rows    seal_rows / open_ghash_rows / ctr_rows (tiles.cuh): how a
               tile's J rows split into generic edge rows and the check-free
               interior loop;
  grids        horner_grid and the open-CTR rows_per_cta split
               (gpu_aesgcm.cu), which cut one object into tiles;
  batch plan   batch_plan_kernel (batch.cuh): tile height J*, per-object
               (J, G) and the tile queue order.
The interior loops index memory without bounds checks, so these replays are
their bounds proofs.
"""

from __future__ import annotations

T = 512              # kHornerThreads == kCtrThreads
SEAL_PAIR = 2        # rows per interior iteration of seal_rows
OPEN_R = 2           # kOpenChains: rows per interior iteration of open_ghash_rows
CTR_PAIR = 2
BATCH_WAVES = 8      # kBatchWaves
BATCH_MAX_SMS = 256  # kBatchMaxSms
PLAN_CANDIDATES = 16  # kPlanCandidates
SMALL_MAX_BLOCKS = 1024  # kSmallMaxBlocks
TILE_OVERHEAD_ROWS = 4.0  # kTileOverheadRows
BATCH_EXTRA = BATCH_WAVES * BATCH_MAX_SMS


def cdiv(a, b):
    return -(-a // b)


def _trunc_div(a, b):
    """C++ integer division (truncates toward zero)."""
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b > 0) else -q


def pad_rows(base):
    """Leading rows of a tile that hold no block of the object (skipped)."""
    return _trunc_div(-base, T) if base < 0 else 0


def _split(pad, r_a, n_interior, rows):
    """The row loops of the tile functions: r runs from the first non-padding
    row up to r_a (generic), then the interior rows [r_a, r_a + n_interior)
    when there are any, then generic rows from wherever r stands to `rows`."""
    generic = list(range(pad, r_a))
    r = max(pad, r_a)
    interior = []
    if n_interior > 0:
        interior = list(range(r_a, r_a + n_interior))
        r = r_a + n_interior
    generic += list(range(r, rows))
    return generic, interior


def seal_tile_rows(base, rows, P, pt_aligned=True):
    """(generic rows, interior rows) of seal_rows for a tile. A misaligned
    plaintext reads the two aligned chunks around a block, so its interior
    blocks are 1 .. n_full - 2."""
    n_full = P // 16
    lo_block = 0 if pt_aligned else 1
    r_lo = 0 if base >= lo_block else _trunc_div(lo_block - base + T - 1, T)
    r_hi = min(_trunc_div(n_full - (0 if pt_aligned else 1) - base, T), rows)
    r_a = min(_trunc_div(r_lo + SEAL_PAIR - 1, SEAL_PAIR) * SEAL_PAIR, r_hi)
    ngroups = _trunc_div(r_hi - r_a, SEAL_PAIR) if r_hi > r_a else 0
    return _split(pad_rows(base), r_a, SEAL_PAIR * ngroups, rows)


def open_tile_rows(base, rows, P):
    """(generic rows, interior rows) of open_ghash_rows for a tile."""
    n_full = P // 16
    r_lo = 0 if base >= 1 else _trunc_div(1 - base + T - 1, T)
    r_hi = min(_trunc_div(n_full - base, T), rows)
    r_a = min(_trunc_div(r_lo + OPEN_R - 1, OPEN_R) * OPEN_R, r_hi)
    ngroups = _trunc_div(r_hi - r_a, OPEN_R) if r_hi > r_a else 0
    return _split(pad_rows(base), r_a, OPEN_R * ngroups, rows)


def ctr_tile_rows(base, rows, P):
    """(generic rows, interior rows) of ctr_rows for a tile."""
    n_full = P // 16
    r_lo = 0 if base >= 1 else _trunc_div(1 - base + T - 1, T)
    r_hi = min(_trunc_div(n_full - base, T), rows)
    if r_lo > r_hi:
        r_lo = r_hi = rows
    npair = _trunc_div(r_hi - r_lo, CTR_PAIR)
    return _split(pad_rows(base), r_lo, CTR_PAIR * npair, rows)


def horner_grid(n, sms):
    j = max(1, cdiv(n, sms * T))
    return j, cdiv(n, j * T)


def ctr_grid(n, sms):
    rows_total = cdiv(n, T)
    per = cdiv(rows_total, sms)
    return per, cdiv(rows_total, per)


def tile_base(n, J, G, c):
    """First block of tile c of G (J rows each), tiles aligned to the end."""
    return n - (G - c) * J * T


def plan_tile_height(rows, sms, count):
    """Tile height J* of batch_plan_kernel (rows: per object, 0 = invalid)."""
    R = sum(rows)
    max_rows = max(rows) if rows else 0
    cand = []
    for c in range(PLAN_CANDIDATES):
        if c < 8:
            j = cdiv(R, (c + 1) * sms)
        else:
            j = cdiv(max_rows, c - 7)
        j = min(j, max_rows)
        cand.append(max(1, j))
    tiles = [sum((1 if r <= J else cdiv(r, J)) for r in rows if r) for J in cand]
    best, best_est = -1, 0.0
    for c in range(PLAN_CANDIDATES):
        t = tiles[c]
        if t == 0 or t > count + BATCH_EXTRA:
            continue
        est = float(cdiv(t, sms)) * (float(R) / float(t) + TILE_OVERHEAD_ROWS)
        if best < 0 or est < best_est or (est == best_est and cand[c] > cand[best]):
            best, best_est = c, est
    return 1 if best < 0 else cand[best]


def batch_plan(lens, sms, valid=None):
    """batch_plan_kernel: returns (jstar, [(J, G), or None for an invalid or
    small object, per object], queue) where the queue lists (object, tile) in
    device order up to the order inside one bucket (the device fills a bucket
    with atomics)."""
    count = len(lens)
    valid = valid if valid is not None else [True] * count
    rows = []
    for P, ok in zip(lens, valid):
        n = cdiv(P, 16)
        # objects of at most SMALL_MAX_BLOCKS blocks take the warp-per-object
        # path and get no tiles
        rows.append(cdiv(n, T) if ok and n > SMALL_MAX_BLOCKS else 0)
    sms = min(sms, BATCH_MAX_SMS)
    jstar = plan_tile_height(rows, sms, count)
    plan = []
    buckets = {}
    for i, (P, r) in enumerate(zip(lens, rows)):
        if r == 0:
            plan.append(None)
            continue
        J = min(r, jstar)
        n = cdiv(P, 16)
        G = max(1, cdiv(n, J * T))
        plan.append((J, G))
        buckets.setdefault(J.bit_length() - 1, []).extend((i, c) for c in range(G))
    queue = [t for b in sorted(buckets, reverse=True) for t in buckets[b]]
    return jstar, plan, queue
