"""CPU replays of the kernels' index arithmetic (test infrastructure).

Each function restates, line for line, one piece of confkv_b200/csrc:
  tile rows    seal_rows / open_ghash_rows / ctr_rows (tiles.cuh): how a
               tile's J rows split into generic edge rows and the check-free
               interior loop;
  grids        horner_grid and the open-CTR rows_per_cta split
               (gpu_aesgcm.cu), which cut one object into tiles;
  batch plan   batch_plan_kernel (batch.cuh): which objects take one warp
               each, the row space of the tile objects, its chunks and each
               chunk's segments.
The interior loops index memory without bounds checks, so these replays are
their bounds proofs.
"""

from __future__ import annotations

T = 512              # kHornerThreads == kCtrThreads
SEAL_PAIR = 2        # rows per interior iteration of seal_rows
OPEN_R = 2           # kOpenChains: rows per interior group of the per-object open_ghash_rows
OPEN_BATCH_R = 4     # kOpenBatchChains: the same for the batched GHASH passes
CTR_PAIR = 2
BATCH_MAX_SMS = 256  # kBatchMaxSms
CHUNKS_PER_SM = 4    # kChunksPerSm
CHUNKS_PER_SM_FEW = 1  # kChunksPerSmFew
MIN_CHUNK_ROWS = 64  # kMinChunkRows
MAX_CHUNKS = CHUNKS_PER_SM * BATCH_MAX_SMS
SMALL_MAX_BLOCKS = 1024  # kSmallMaxBlocks
WARP_MAX_BLOCKS = 2048   # kWarpMaxBlocks
MID_ALPHA_SEAL = 26      # kMidAlphaSeal
MID_ALPHA_OPEN = 19      # kMidAlphaOpen
SEGMENT_COST_ROWS = 5    # kSegmentCostRows
UNIFORM_ROWS_RATIO = 2   # kUniformRowsRatio


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
    # one GHASH chain (kSealChains = 1): the two-row loop starts at r_lo
    r_a = min(r_lo, r_hi)
    ngroups = _trunc_div(r_hi - r_a, SEAL_PAIR) if r_hi > r_a else 0
    return _split(pad_rows(base), r_a, SEAL_PAIR * ngroups, rows)


def open_tile_rows(base, rows, P, R=OPEN_R):
    """(generic rows, interior rows) of open_ghash_rows with R chains for a tile."""
    n_full = P // 16
    r_lo = 0 if base >= 1 else _trunc_div(1 - base + T - 1, T)
    r_hi = min(_trunc_div(n_full - base, T), rows)
    r_a = min(_trunc_div(r_lo + R - 1, R) * R, r_hi)
    ngroups = _trunc_div(r_hi - r_a, R) if r_hi > r_a else 0
    return _split(pad_rows(base), r_a, R * ngroups, rows)


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


def chunk_count(R, K, sms, uniform=False):
    """batch_chunk_count: chunks for R rows of K tile objects on `sms` SMs
    (`uniform`: the largest tile or mid object has at most UNIFORM_ROWS_RATIO
    times the rows of the smallest)."""
    if R == 0:
        return 0
    cap = CHUNKS_PER_SM if K >= CHUNKS_PER_SM * sms and not uniform else CHUNKS_PER_SM_FEW
    per = max(1, min(cap, R // (sms * MIN_CHUNK_ROWS)))
    return min(per * sms, R)


def chunk_row(c, R, M):
    return c * R // M


def chunk_of(x, R, M):
    return ((x + 1) * M - 1) // R


def tile_rows(P, ok=True, mid_routed=False):
    """Rows of a tile object (0 for small and invalid objects, and for mid
    objects when the batch sends them down the warp path)."""
    n = cdiv(P, 16)
    if not ok or n <= SMALL_MAX_BLOCKS or (mid_routed and n <= WARP_MAX_BLOCKS):
        return 0
    return cdiv(n, T)


def mid_routed(lens, sms, valid=None, open_=False):
    """The plan's routing rule: mid objects (SMALL_MAX_BLOCKS + 1 ..
    WARP_MAX_BLOCKS blocks) take one warp each when there are any and the
    batch's N warp-path objects (small plus mid) satisfy
    N * sum(rows + o) * T >= alpha * max_n * sms * mids over the mid
    objects; `sms` is the plan's SM count (at most BATCH_MAX_SMS)."""
    valid = valid if valid is not None else [True] * len(lens)
    blocks = [cdiv(P, 16) for P, ok in zip(lens, valid) if ok]
    mid = [n for n in blocks if SMALL_MAX_BLOCKS < n <= WARP_MAX_BLOCKS]
    if not mid:
        return False
    warp = sum(1 for n in blocks if n <= WARP_MAX_BLOCKS)
    cost = sum(cdiv(n, T) + SEGMENT_COST_ROWS for n in mid)
    alpha = MID_ALPHA_OPEN if open_ else MID_ALPHA_SEAL
    return warp * cost * T >= alpha * max(mid) * sms * len(mid)


def chunk_plan(lens, sms, valid=None, classes=None, open_=False):
    """batch_plan_kernel: the row space (tile objects grouped by alignment
    class; inside a class the device order follows its atomics, here the
    descriptor order), its chunk count M, the chunks' first rows (cut at
    equal cost, a tile object weighing its rows plus SEGMENT_COST_ROWS), the
    first tile object of each chunk and the segment count of each object (0
    for small and invalid ones)."""
    valid = valid if valid is not None else [True] * len(lens)
    classes = classes if classes is not None else [0] * len(lens)
    sms = min(sms, BATCH_MAX_SMS)
    routed = mid_routed(lens, sms, valid, open_)
    objs, row = [], 0
    order = sorted(range(len(lens)), key=lambda i: (classes[i], i))
    for i in order:
        rows = tile_rows(lens[i], valid[i], routed)
        if rows:
            objs.append((row, i, rows))
            row += rows
    R, K = row, len(objs)
    sized = [tile_rows(P, ok) for P, ok in zip(lens, valid)]   # tile and mid objects, before routing
    sized = [r for r in sized if r]
    uniform = K != 0 and max(sized) <= UNIFORM_ROWS_RATIO * min(sized)
    M = chunk_count(R, K, sms, uniform)
    o = SEGMENT_COST_ROWS if M and (R + SEGMENT_COST_ROWS * K) // M >= 2 * (SEGMENT_COST_ROWS + 1) else 0
    C = R + o * K
    chunk_first = [None] * M
    chunk_start = [None] * M + [R]
    segs = [0] * len(lens)
    for k, (start, i, rows) in enumerate(objs):
        p = start + o * k
        first, last = chunk_of(p + o, C, M), chunk_of(p + o + rows - 1, C, M)
        segs[i] = last - first + 1
        c = chunk_of(p, C, M)
        c = c if chunk_row(c, C, M) == p else c + 1
        for c in range(c, last + 1):
            assert chunk_first[c] is None
            x = chunk_row(c, C, M)
            chunk_first[c] = k
            chunk_start[c] = start + max(0, x - p - o)
    return {"R": R, "M": M, "objs": objs, "chunk_first": chunk_first, "chunk_start": chunk_start,
            "segments": segs, "mid_routed": routed}


def chunk_segments(plan, chunk):
    """Segments of one chunk as the work kernels walk them (Cursor,
    segment_at, cursor_step): (item, rows, r0, r1) each."""
    objs = plan["objs"]
    a0, b = plan["chunk_start"][chunk], plan["chunk_start"][chunk + 1]
    k = plan["chunk_first"][chunk]
    out = []
    while True:
        start, item, rows = objs[k]
        end = start + rows
        a = max(a0, start)
        out.append((item, rows, a - start, min(b, end) - start))
        if end >= b:
            return out
        k += 1


def segment_base(P, rows, r0):
    """First block of a segment starting at row r0 of an object of `rows` rows."""
    return cdiv(P, 16) - (rows - r0) * T
