// Batched seal / open: one plan launch and one (seal) or two (open)
// persistent launches for any number of objects of any sizes and alignments.
//
//   batch_plan_kernel    one CTA: validates every descriptor (status), sums
//                        the rows, picks the tile height J* by scoring 16
//                        candidates (1..8 tiles per SM, the tallest object
//                        in 1..8 equal tiles) with a makespan model, gives object i
//                        J_i = min(J*, rows_i) and G_i = ceil(n_i / (J_i T))
//                        tiles, and writes the tile records (object, tile)
//                        with taller tiles first, so the queue's tail holds
//                        the short ones.
//   seal_batch_kernel    one CTA per SM; each takes tiles from the queue
//   open_ghash_batch_    (atomic head) and runs the same tile bodies as the
//   kernel               single-object kernels (tiles.cuh). A one-tile
//   open_ctr_batch_      object needs no atomics; others accumulate through
//   kernel               their slot and the last tile writes the tag / the
//                        verdict. No CTA waits for another.
//
// Device-written workspace (caller-owned, any contents on entry):
//   [0, 256)            BatchHeader
//   [256, ...)          one Slot per object: acc, ticket, aux = {J, G, verdict}
//   [tiles_offset, ...) TileRec per tile, at most count + kBatchExtraTiles
//   [small_offset, ...) small objects (item indices), largest first
#pragma once

#include "small.cuh"
#include "tiles.cuh"

namespace confkv {
namespace dev {


constexpr int kBatchWaves = 8;        // most tiles per SM the plan considers
constexpr int kPlanCandidates = 16;   // tile heights the plan scores
// Fixed work per tile (fold, tag or verdict, table refill, queue and
// descriptor fetch) in units of one row of the seal loop, as measured on
// B200: about 8-10 us per tile against ~2.5 us per 8 KiB row per SM.
constexpr double kTileOverheadRows = 4.0;
constexpr int kBatchMaxSms = 256;     // SMs counted for the tile bound
constexpr uint32_t kBatchExtraTiles = static_cast<uint32_t>(kBatchWaves * kBatchMaxSms);
constexpr uint32_t kBatchMaxItems = 1u << 20;
constexpr int kPlanThreads = 1024;
constexpr int kBuckets = 32;
constexpr uint64_t kBatchMaxBlocks = 0xfffffffeull;
constexpr uint32_t kCtrBatchMisc = kSmallSmem;      // after the small-object tables
constexpr uint32_t kCtrBatchSmem = kCtrBatchMisc + 64;
constexpr int kSmallBuckets = 11;                   // floor(log2 n) of a small object, n <= 1024

// Hand-off from the row warps to the power warp (two-stage fold, tiles.cuh):
// two buffers of 32 partials, and per buffer a FULL mbarrier (the 16 row
// warps arrived) and an EMPTY one (the power warp took the values).
constexpr uint32_t kHandoffBytes = 2 * 32 * 16;
constexpr uint32_t kHandoffSyncBytes = 64;
// Batched seal shared memory: AES tables, the chain table H^512 (H^32 for
// small objects), the row-warp fold tables H^8, H^1, H^2, H^4 (the slots the
// small-object path reads), the hand-off buffers and their mbarriers.
constexpr uint32_t kSealBatchFold = kAesBytes + kGhBytes;
constexpr uint32_t kSealBatchHandoff = kSealBatchFold + 4 * 8192u;
constexpr uint32_t kSealBatchSync = kSealBatchHandoff + kHandoffBytes;
constexpr uint32_t kSealBatchSmem = kSealBatchSync + kHandoffSyncBytes;
static_assert(kSealBatchFold == kSmallFold, "the small-object path reads the seal fold slots");
static_assert(kSealBatchSmem <= 227u * 1024u, "batched seal shared memory exceeds the per-block limit");
// Batched open-GHASH shared memory: the single-object layout up to the
// compact H^512 table, then the hand-off.
constexpr uint32_t kOpenBatchHandoff = kOpenHt + 8192u;
constexpr uint32_t kOpenBatchSync = kOpenBatchHandoff + kHandoffBytes;
constexpr uint32_t kOpenBatchSmem = kOpenBatchSync + kHandoffSyncBytes;

// Alignment classes: 2 v + p, v = the frame's ciphertext class (seal: store
// funnel word part 0..3, 4 = aligned; open: load funnel word part, same
// coding) and p = 1 when the plaintext side (seal src, open dst) is 16-B
// aligned. Each tile record carries its object's class; the work kernels run
// a loop specialised for it and switch loops only when the class changes.
constexpr int kClasses = 10;

struct BatchHeader {
    uint32_t total_tiles;
    uint32_t next_tile[2];   // queue heads: [0] seal / open GHASH, [1] open CTR
    uint32_t iters_max;      // J*
    uint32_t small_count;    // objects of at most kSmallMaxBlocks blocks, one warp each
    uint32_t small_next[2];  // small-object queue heads: [0] seal, [1] open
    uint32_t fault;          // nonzero: a work kernel's hand-off wait gave up (results invalid)
    uint32_t pad[8];
};
static_assert(sizeof(BatchHeader) <= 256, "batch header fits its 256-byte area");

struct TileRec {
    uint32_t item;
    uint32_t cta;            // tile index c within the object (bits 0-23) | class << 24
};
constexpr uint32_t kTileIndexMask = 0x00ffffffu;

__host__ __device__ constexpr size_t batch_slots_offset() { return 256; }
__host__ __device__ constexpr size_t batch_tiles_offset(size_t count)
{
    return 256 + (count * sizeof(Slot) + 255) / 256 * 256;
}
__host__ __device__ constexpr size_t batch_small_offset(size_t count)
{
    return batch_tiles_offset(count) + (count + kBatchExtraTiles) * sizeof(TileRec);
}
__host__ __device__ constexpr size_t batch_workspace_bytes(size_t count)
{
    return batch_small_offset(count) + count * sizeof(uint32_t);
}

struct BatchArgs {
    BatchItem* items;
    uint8_t* ws;
    uint32_t count;
    uint32_t rk[44];
    KeyTables kt;
};

// Ciphertext store class of a frame: sq = word part of 16 - (ct & 15)
// (4 when aligned), r = its byte part.
__device__ __forceinline__ void store_class(const uint8_t* ct, int& sq, uint32_t& r)
{
    const uint32_t off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(ct) & 15u);
    sq = 4;
    r = 0;
    if (off != 0) {
        const uint32_t sh = 16u - off;
        sq = static_cast<int>(sh >> 2);
        r = sh & 3u;
    }
}

// Ciphertext load class of a frame: lq = word part of (ct & 15) (4 when
// aligned), r = its byte part.
__device__ __forceinline__ void load_class(const uint8_t* ct, int& lq, uint32_t& r)
{
    const uint32_t off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(ct) & 15u);
    lq = off == 0 ? 4 : static_cast<int>(off >> 2);
    r = off & 3u;
}

__device__ __forceinline__ int item_class(const BatchItem& it, int open)
{
    int v;
    uint32_t r;
    if (open) {
        load_class(it.src + 13, v, r);
        return 2 * v + ((reinterpret_cast<uintptr_t>(it.dst) & 15u) == 0);
    }
    store_class(it.dst + 13, v, r);
    return 2 * v + ((reinterpret_cast<uintptr_t>(it.src) & 15u) == 0);
}

// ------------------------------------------------------------------ plan

// `open` selects the descriptor rules: seal needs capacity >= P + 29; open
// needs frame length >= P + 29 and an auth_ok pointer. sms = SMs the work
// kernels run on (at most kBatchMaxSms).
__global__ void __launch_bounds__(kPlanThreads) batch_plan_kernel(BatchItem* items, uint32_t count,
                                                                  uint8_t* ws, int open, uint32_t sms)
{
    __shared__ unsigned long long red[kPlanThreads / 32];
    __shared__ uint32_t red_max[kPlanThreads / 32];
    __shared__ unsigned int hist[kBuckets][kClasses];
    __shared__ unsigned int cursor[kBuckets][kClasses];
    __shared__ unsigned long long total_rows;
    __shared__ uint32_t max_rows;
    __shared__ uint32_t cand[kPlanCandidates];
    __shared__ unsigned long long cand_tiles[kPlanCandidates];
    __shared__ uint32_t cand_part[kPlanThreads / 32][kPlanCandidates];
    __shared__ uint32_t jstar_s;
    __shared__ unsigned int small_hist[kSmallBuckets];
    __shared__ unsigned int small_cursor[kSmallBuckets];
    BatchHeader* hdr = reinterpret_cast<BatchHeader*>(ws);
    uint32_t* small_list = reinterpret_cast<uint32_t*>(ws + batch_small_offset(count));
    Slot* st = reinterpret_cast<Slot*>(ws + batch_slots_offset());
    TileRec* rec = reinterpret_cast<TileRec*>(ws + batch_tiles_offset(count));
    const int tid = threadIdx.x;
    constexpr uint64_t T = kHornerThreads;
    pdl_release();
    for (int i = tid; i < kClasses * kBuckets; i += kPlanThreads) {
        hist[i / kClasses][i % kClasses] = 0;
    }
    if (tid < kSmallBuckets) {
        small_hist[tid] = 0;
    }
    __syncthreads();
    pdl_wait();  // descriptors and workspace may belong to earlier work on the stream

    // Pass 1: validate, rows per object (a zero-length object is one row:
    // its tile writes the header and tag), reset the slot.
    unsigned long long rows_sum = 0;
    uint32_t rows_max = 0;
    for (uint32_t i = tid; i < count; i += kPlanThreads) {
        BatchItem& it = items[i];
        const uint64_t P = it.plen;
        const uint64_t n = P / 16u + ((P & 15u) != 0);
        bool ok = it.src != nullptr && it.dst != nullptr && n <= kBatchMaxBlocks && it.capacity >= P + 29u;
        if (open) {
            ok = ok && it.auth_ok != nullptr;
        }
        // small objects go to the warp-per-object list (aux[2] = bucket + 1),
        // the others to the tile planner (aux[0] = rows)
        const bool small = ok && n <= kSmallMaxBlocks;
        const uint32_t rows = ok && !small ? static_cast<uint32_t>((n + T - 1) / T) : 0u;
        it.status = ok ? 0 : -1;
        Slot& s = st[i];
        s.acc_hi = 0;
        s.acc_lo = 0;
        s.ticket = 0;
        s.aux[0] = rows;
        s.aux[1] = 0;
        s.aux[2] = 0;
        if (small) {
            const int b = 31 - __clz(static_cast<int>(n | 1u));
            s.aux[2] = static_cast<uint32_t>(b + 1);
            atomicAdd(&small_hist[b], 1u);
        }
        rows_sum += rows;
        rows_max = rows > rows_max ? rows : rows_max;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        rows_sum += __shfl_xor_sync(0xffffffffu, rows_sum, o);
        const uint32_t m = __shfl_xor_sync(0xffffffffu, rows_max, o);
        rows_max = m > rows_max ? m : rows_max;
    }
    if ((tid & 31) == 0) {
        red[tid >> 5] = rows_sum;
        red_max[tid >> 5] = rows_max;
    }
    __syncthreads();
    if (tid < 32) {
        unsigned long long v = red[tid];
        uint32_t m = red_max[tid];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            v += __shfl_xor_sync(0xffffffffu, v, o);
            const uint32_t mo = __shfl_xor_sync(0xffffffffu, m, o);
            m = mo > m ? mo : m;
        }
        if (tid == 0) {
            total_rows = v;
            max_rows = m;
        }
    }
    __syncthreads();

    // Tile height J*. Candidates: the heights giving w = 1..8 tiles per SM
    // (ceil(R / (w sms))) and the heights cutting the tallest object into
    // k = 1..8 equal tiles (ceil(max_rows / k)). Each is scored by the
    // makespan of equal tiles on `sms` SMs, ceil(tiles / sms) x (R / tiles +
    // kTileOverheadRows), among those whose tile count fits the record area
    // (the w = 8 height always does); ties go to the taller tile.
    const unsigned long long R = total_rows;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // Tile counts per candidate: every thread counts its own objects for all
    // candidates, then a warp shuffle reduction and a sum over the warps.
    if (tid < kPlanCandidates) {
        unsigned long long j;
        if (tid < 8) {
            const unsigned long long slots = static_cast<unsigned long long>(tid + 1) * sms;
            j = (R + slots - 1) / slots;
        } else {
            const uint32_t k = static_cast<uint32_t>(tid - 7);
            j = (max_rows + k - 1) / k;
        }
        j = j > max_rows ? max_rows : j;
        cand[tid] = static_cast<uint32_t>(j < 1 ? 1 : j);
    }
    __syncthreads();
    {
        uint32_t loc[kPlanCandidates];
#pragma unroll
        for (int c = 0; c < kPlanCandidates; ++c) {
            loc[c] = 0;
        }
        for (uint32_t i = tid; i < count; i += kPlanThreads) {
            const uint32_t rows = st[i].aux[0];
            if (rows == 0) {
                continue;
            }
#pragma unroll
            for (int c = 0; c < kPlanCandidates; ++c) {
                const uint32_t J = cand[c];
                loc[c] += rows <= J ? 1u : (rows + J - 1) / J;
            }
        }
#pragma unroll
        for (int c = 0; c < kPlanCandidates; ++c) {
            uint32_t v = loc[c];
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                v += __shfl_xor_sync(0xffffffffu, v, o);
            }
            if (lane == 0) {
                cand_part[warp][c] = v;
            }
        }
    }
    __syncthreads();
    if (tid < kPlanCandidates) {
        unsigned long long t = 0;
        for (int w = 0; w < kPlanThreads / 32; ++w) {
            t += cand_part[w][tid];
        }
        cand_tiles[tid] = t;
    }
    __syncthreads();
    // Warp 0 scores the candidates (lane c = candidate c) and keeps the
    // smallest estimate, the taller tile on a tie.
    if (warp == 0) {
        int valid = 0;
        double est = 0.0;
        uint32_t J = 1;
        if (lane < kPlanCandidates) {
            const unsigned long long tiles = cand_tiles[lane];
            J = cand[lane];
            valid = tiles != 0 && tiles <= static_cast<unsigned long long>(count) + kBatchExtraTiles ? 1 : 0;
            if (valid) {
                const double waves = static_cast<double>((tiles + sms - 1) / sms);
                est = waves * (static_cast<double>(R) / static_cast<double>(tiles) + kTileOverheadRows);
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const int ov = __shfl_xor_sync(0xffffffffu, valid, o);
            const double oe = __shfl_xor_sync(0xffffffffu, est, o);
            const uint32_t oj = __shfl_xor_sync(0xffffffffu, J, o);
            if (ov && (!valid || oe < est || (oe == est && oj > J))) {
                valid = 1;
                est = oe;
                J = oj;
            }
        }
        if (lane == 0) {
            jstar_s = valid ? J : 1u;
        }
    }
    __syncthreads();
    const uint32_t jstar = jstar_s;

    // Pass 2: tile height and count per object; histogram of tiles by
    // (alignment class, floor(log2 J)).
    for (uint32_t i = tid; i < count; i += kPlanThreads) {
        Slot& s = st[i];
        const uint32_t rows = s.aux[0];
        if (rows == 0) {
            continue;
        }
        const uint32_t J = rows < jstar ? rows : jstar;
        const uint64_t P = items[i].plen;
        const uint64_t n = P / 16u + ((P & 15u) != 0);
        const uint64_t span = static_cast<uint64_t>(J) * T;
        uint64_t G = (n + span - 1) / span;
        G = G < 1 ? 1 : G;
        s.aux[0] = J;
        s.aux[1] = static_cast<uint32_t>(G);
        atomicAdd(&hist[31 - __clz(static_cast<int>(J))][item_class(items[i], open)], static_cast<unsigned int>(G));
    }
    __syncthreads();
    // Records: tallest bucket first, classes in order inside a bucket (so
    // the queue ends on short tiles and neighbouring tiles share a class).
    // Warp 0: lane l owns bucket 31 - l; an exclusive scan over the lanes
    // gives each bucket's start.
    static_assert(kBuckets == 32, "one lane per height bucket");
    if (warp == 0) {
        const int b = kBuckets - 1 - lane;
        unsigned int total = 0;
#pragma unroll
        for (int c = 0; c < kClasses; ++c) {
            total += hist[b][c];
        }
        unsigned int incl = total;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) {
                incl += v;
            }
        }
        unsigned int pos = incl - total;
#pragma unroll
        for (int c = 0; c < kClasses; ++c) {
            cursor[b][c] = pos;
            pos += hist[b][c];
        }
        if (lane == 31) {
            hdr->total_tiles = incl;
            hdr->next_tile[0] = 0;
            hdr->next_tile[1] = 0;
            hdr->iters_max = jstar;
            hdr->fault = 0;
        }
    } else if (warp == 1 && lane == 0) {
        // small objects: largest bucket first
        unsigned int pos = 0;
        for (int b = kSmallBuckets - 1; b >= 0; --b) {
            small_cursor[b] = pos;
            pos += small_hist[b];
        }
        hdr->small_count = pos;
        hdr->small_next[0] = 0;
        hdr->small_next[1] = 0;
    }
    __syncthreads();

    // Pass 3: tile records and the small-object list.
    for (uint32_t i = tid; i < count; i += kPlanThreads) {
        const Slot& s = st[i];
        const uint32_t G = s.aux[1];
        if (G == 0) {
            if (s.aux[2] != 0 && s.aux[0] == 0) {
                small_list[atomicAdd(&small_cursor[s.aux[2] - 1], 1u)] = i;
            }
            continue;
        }
        const uint32_t cls = static_cast<uint32_t>(item_class(items[i], open));
        const unsigned int p = atomicAdd(&cursor[31 - __clz(static_cast<int>(s.aux[0]))][cls], G);
        for (uint32_t c = 0; c < G; ++c) {
            rec[p + c] = TileRec{i, c | (cls << 24)};
        }
    }
}

// Final GHASH sum of a tile's object: a one-tile object multiplies its fold
// by H^2 directly; otherwise the fold goes through the object's slot and only
// the last tile gets the sum. Power warp only; returns true where (shi, slo)
// holds the sum.
__device__ __forceinline__ bool batch_object_sum(Slot* slot, uint32_t G, uint4 fold, unsigned long long uhi,
                                                 unsigned long long ulo, int lane, unsigned long long& shi,
                                                 unsigned long long& slo)
{
    if (G == 1) {
        warp_generic_mul(fold, uhi, ulo, lane, shi, slo);
        return true;
    }
    return cta_accumulate(slot, fold, uhi, ulo, lane, G, shi, slo);
}

// Shared state of the work kernels: the workspace views and the CTA's
// coordinates.
struct BatchCta {
    BatchHeader* hdr;
    Slot* st;
    const TileRec* rec;
    uint32_t total;
    int tid;
    int lane;
    int warp;
};

__device__ __forceinline__ int tile_class(const BatchCta& c, uint32_t tile)
{
    return static_cast<int>(c.rec[tile].cta >> 24);
}

// First queue index of this CTA (all threads); the barriers bracket the
// shared broadcast.
__device__ __forceinline__ uint32_t first_tile(volatile uint32_t* next_s, const BatchCta& c, int pass)
{
    if (c.tid == 0) {
        *next_s = atomicAdd(&c.hdr->next_tile[pass], 1u);
    }
    __syncthreads();
    const uint32_t t = *next_s;
    __syncthreads();
    return t;
}

// ------------------------------------------------------------- hand-off
//
// Seal and open-GHASH CTAs run their tiles as a pipeline: the 16 row warps
// compute a tile's rows and the first fold stage, hand 32 values to the power
// warp and go on with the next tile, while the power warp finishes the fold,
// the object's sum and the tag (seal) or verdict (open). Hand-off j uses
// buffer j & 1; its FULL mbarrier completes when the 16 row warps arrived,
// its EMPTY mbarrier when the power warp has read the values, so a buffer is
// rewritten only after it was read. Both sides take the tiles in the same
// queue order: thread 0 takes the next index after its rows and passes it
// along with the values.

// Shared-memory views of the hand-off (kHandoffBytes of buffers at part_off,
// kHandoffSyncBytes of mbarriers and words at sync_off).
struct Handoff {
    uint4* part;               // [2][32] fold values V_p
    uint64_t* full;            // [2]
    uint64_t* empty;           // [2]
    volatile uint32_t* next;   // [2] queue index taken after the buffer's tile
    volatile uint32_t* first;  // first queue index of the CTA
    volatile uint32_t* abort;  // raised by a wait that gave up
};

__device__ __forceinline__ Handoff handoff_at(uint8_t* smem, uint32_t part_off, uint32_t sync_off)
{
    uint8_t* s = smem + sync_off;
    return Handoff{reinterpret_cast<uint4*>(smem + part_off), reinterpret_cast<uint64_t*>(s),
                   reinterpret_cast<uint64_t*>(s + 16), reinterpret_cast<volatile uint32_t*>(s + 32),
                   reinterpret_cast<volatile uint32_t*>(s + 40), reinterpret_cast<volatile uint32_t*>(s + 44)};
}

// Thread 0, before the CTA's first barrier.
__device__ __forceinline__ void handoff_init(const Handoff& h)
{
    mbar_init(h.full, kHornerThreads / 32);
    mbar_init(h.full + 1, kHornerThreads / 32);
    mbar_init(h.empty, 1);
    mbar_init(h.empty + 1, 1);
    *h.abort = 0u;
}

// Row warps, hand-off j: wait until the power warp has read the buffer's
// previous values (the first use of each buffer passes at once), store the
// warp's V_2w and V_2w+1 and, thread 0, the queue index it took, arrive, and
// wait for the other row warps so that every thread reads the next index.
// False, in the whole warp, when a wait gave up.
__device__ __forceinline__ bool row_handoff(const Handoff& h, uint32_t j, uint4 v, uint32_t taken,
                                            const BatchCta& c, uint32_t& next)
{
    const uint32_t b = j & 1u;
    const uint32_t parity = (j >> 1) & 1u;
    if (!__all_sync(0xffffffffu, mbar_wait(h.empty + b, parity ^ 1u, h.abort))) {
        return false;
    }
    if (c.lane < 2) {
        h.part[32 * b + 2 * c.warp + c.lane] = v;
    }
    if (c.tid == 0) {
        h.next[b] = taken;
    }
    __syncwarp();
    if (c.lane == 0) {
        mbar_arrive(h.full + b);
    }
    if (!__all_sync(0xffffffffu, mbar_wait(h.full + b, parity, h.abort))) {
        return false;
    }
    next = h.next[b];
    return true;
}

// Power warp, hand-off j: wait for the row warps' values (lane p takes V_p)
// and the next queue index, then free the buffer.
__device__ __forceinline__ bool power_take(const Handoff& h, uint32_t j, int lane, uint4& v, uint32_t& next)
{
    const uint32_t b = j & 1u;
    if (!__all_sync(0xffffffffu, mbar_wait(h.full + b, (j >> 1) & 1u, h.abort))) {
        return false;
    }
    v = h.part[32 * b + lane];
    next = h.next[b];
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(h.empty + b);
    }
    return true;
}

// Work-kernel epilogue of the tile phase (all threads): a CTA whose hand-off
// gave up marks the batch as faulted and reports true.
__device__ __forceinline__ bool handoff_failed(const Handoff& h, const BatchCta& c)
{
    __syncthreads();
    if (*h.abort == 0u) {
        return false;
    }
    if (c.tid == 0) {
        atomicOr(&c.hdr->fault, 1u);
    }
    return true;
}

// ------------------------------------------------------------------ seal

// Row warps: tiles of one alignment class, from `tile` while the queue hands
// out tiles of this class; returns the first tile of another class (or >=
// total). Per-tile values are loaded where they are used so that only the
// tile index stays live across the rows.
template <int SQ, bool PT>
__device__ __forceinline__ uint32_t seal_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c,
                                               const Handoff& h, uint32_t tile, int cls, uint32_t& j)
{
    constexpr int64_t T = kHornerThreads;
    const uint4* ft = reinterpret_cast<const uint4*>(smem + kSealBatchFold);
    for (;;) {
        uint4 q;
        {
            const TileRec tr = c.rec[tile];
            const uint32_t cta = tr.cta & kTileIndexMask;
            const BatchItem* it = a.items + tr.item;
            const uint32_t J = c.st[tr.item].aux[0];
            const uint32_t G = c.st[tr.item].aux[1];
            const uint64_t P = it->plen;
            const int64_t n = static_cast<int64_t>(P / 16u + ((P & 15u) != 0));
            const int64_t span = static_cast<int64_t>(J) * T;
            uint8_t* frame = it->dst;
            const uint32_t ivw[3] = {it->iv[0], it->iv[1], it->iv[2]};
            if (cta == 0 && c.tid == 0) {
                frame[0] = 1;
                for (int b = 0; b < 12; ++b) {
                    frame[1 + b] = static_cast<uint8_t>(ivw[b >> 2] >> (8 * (b & 3)));
                }
            }
            int sq;
            uint32_t store_r;
            store_class(frame + 13, sq, store_r);  // sq == SQ for this class
            (void)sq;
            const SealTile t{it->src, frame + 13, P, n - static_cast<int64_t>(G - cta) * span,
                             static_cast<int64_t>(J), {ivw[0] ^ a.rk[0], ivw[1] ^ a.rk[1], ivw[2] ^ a.rk[2]},
                             store_r};
            q = seal_rows<SQ, PT>(t, a.rk, a.kt.gh_pow2, c.tid, c.lane);
        }
        uint32_t taken = 0;
        if (c.tid == 0) {
            taken = atomicAdd(&c.hdr->next_tile[0], 1u);
        }
        const uint4 v = warp_fold_pairs<true>(q, ft, c.lane);
        uint32_t next;
        if (!row_handoff(h, j, v, taken, c, next)) {
            return c.total;
        }
        ++j;
        if (next >= c.total || tile_class(c, next) != cls) {
            return next;
        }
        tile = next;
    }
}

// Power warp of the batched seal, over the same tiles as the row warps:
// E_K(J0), L*H and the basis of H^d while the tile's rows run, then the fold
// levels 4..8 (the key's global tables), the object's sum and, once the
// object's last tile is in, its tag.
__device__ __forceinline__ void seal_power_loop(const BatchArgs& a, const BatchCta& c, const Handoff& h,
                                                uint32_t tile)
{
    constexpr unsigned long long T = kHornerThreads;
    for (uint32_t j = 0; tile < c.total; ++j) {
        const TileRec tr = c.rec[tile];
        const uint32_t cta = tr.cta & kTileIndexMask;
        Slot* slot = c.st + tr.item;
        const BatchItem* it = a.items + tr.item;
        const uint32_t J = slot->aux[0];
        const uint32_t G = slot->aux[1];
        const uint64_t P = it->plen;
        const uint32_t ivw[3] = {it->iv[0], it->iv[1], it->iv[2]};
        const unsigned long long d = static_cast<unsigned long long>(G - 1 - cta) * J * T + 2ull;
        uint4 ej0, lh;
        unsigned long long uhi, ulo;
        seal_power(ivw, a.rk, P, d, a.kt.gh_pow2, c.lane, ej0, lh, uhi, ulo);
        uint4 v;
        uint32_t next;
        if (!power_take(h, j, c.lane, v, next)) {
            return;
        }
        const uint4 fold = power_fold(v, a.kt.gh_pow2 + 4 * 512, c.lane);
        unsigned long long shi, slo;
        if (batch_object_sum(slot, G, fold, uhi, ulo, c.lane, shi, slo)) {
            const uint4 tag = xor4(xor4(be_to_raw(shi, slo), lh), ej0);
            if (c.lane < 16) {
                it->dst[13 + P + c.lane] = static_cast<uint8_t>(byte_of(tag, c.lane));
            }
        }
        tile = next;
    }
}

__global__ void __launch_bounds__(kSealThreads, 1) seal_batch_kernel(const BatchArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x;
    pdl_release();
    fill_aes_smem(smem + kSealAes, a.kt.aes_t);
    fill_gh_smem(smem + kSealGh, a.kt.gh_pow2 + kSealChainLog2 * 512);
    fill_small_fold(smem, a.kt.gh_pow2);
    const Handoff h = handoff_at(smem, kSealBatchHandoff, kSealBatchSync);
    if (tid == 0) {
        handoff_init(h);
    }
    pdl_wait();  // the plan kernel's workspace
    auto* hdr = reinterpret_cast<BatchHeader*>(a.ws);
    const BatchCta c{hdr, reinterpret_cast<Slot*>(a.ws + batch_slots_offset()),
                     reinterpret_cast<const TileRec*>(a.ws + batch_tiles_offset(a.count)), hdr->total_tiles,
                     tid, tid & 31, tid >> 5};
    uint32_t tile = first_tile(h.first, c, 0);
    if (c.warp == kPowerWarp) {
        seal_power_loop(a, c, h, tile);
    } else {
        uint32_t j = 0;
        while (tile < c.total) {
            const int cls = tile_class(c, tile);
            switch (cls) {
            case 0: tile = seal_class<0, false>(smem, a, c, h, tile, cls, j); break;
            case 1: tile = seal_class<0, true>(smem, a, c, h, tile, cls, j); break;
            case 2: tile = seal_class<1, false>(smem, a, c, h, tile, cls, j); break;
            case 3: tile = seal_class<1, true>(smem, a, c, h, tile, cls, j); break;
            case 4: tile = seal_class<2, false>(smem, a, c, h, tile, cls, j); break;
            case 5: tile = seal_class<2, true>(smem, a, c, h, tile, cls, j); break;
            case 6: tile = seal_class<3, false>(smem, a, c, h, tile, cls, j); break;
            case 7: tile = seal_class<3, true>(smem, a, c, h, tile, cls, j); break;
            case 8: tile = seal_class<4, false>(smem, a, c, h, tile, cls, j); break;
            default: tile = seal_class<4, true>(smem, a, c, h, tile, cls, j); break;
            }
        }
    }
    if (handoff_failed(h, c)) {
        return;
    }

    // Small objects, one warp each, once the tiles are gone: H^32 over the
    // chain table (the fold slots already hold H^8, H^1, H^2, H^4).
    const uint32_t small_count = hdr->small_count;
    if (small_count == 0) {
        return;
    }
    fill_gh_smem(smem + kSmallGh, a.kt.gh_pow2 + 5 * 512);
    __syncthreads();
    const uint32_t* small_list = reinterpret_cast<const uint32_t*>(a.ws + batch_small_offset(a.count));
    for (;;) {
        uint32_t k = 0;
        if (c.lane == 0) {
            k = atomicAdd(&hdr->small_next[0], 1u);
        }
        k = __shfl_sync(0xffffffffu, k, 0);
        if (k >= small_count) {
            break;
        }
        seal_object_warp(a.items + small_list[k], a.rk, a.kt.gh_pow2, smem, c.lane);
    }
}

// ------------------------------------------------------------------ open

// Row warps of the GHASH pass: tiles whose frames share load class LQ (both
// plaintext sides); returns the first tile of another load class (or >=
// total).
template <int LQ>
__device__ __forceinline__ uint32_t open_ghash_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c,
                                                     const Handoff& h, uint32_t tile, uint32_t& j)
{
    constexpr int64_t T = kHornerThreads;
    const uint4* ft = reinterpret_cast<const uint4*>(smem + kOpenFold);
    for (;;) {
        uint4 q;
        {
            const TileRec tr = c.rec[tile];
            const uint32_t cta = tr.cta & kTileIndexMask;
            const BatchItem* it = a.items + tr.item;
            const uint32_t J = c.st[tr.item].aux[0];
            const uint32_t G = c.st[tr.item].aux[1];
            const uint64_t P = it->plen;
            const int64_t n = static_cast<int64_t>(P / 16u + ((P & 15u) != 0));
            const int64_t span = static_cast<int64_t>(J) * T;
            const uint8_t* frame = it->src;
            int lq;
            uint32_t load_r;
            load_class(frame + 13, lq, load_r);  // lq == LQ for this class
            (void)lq;
            const OpenTile t{frame, it->capacity, P, n - static_cast<int64_t>(G - cta) * span,
                             static_cast<int64_t>(J), load_r};
            q = open_ghash_rows<LQ>(t, reinterpret_cast<const uint4*>(smem + kOpenHt), c.tid, c.lane);
        }
        uint32_t taken = 0;
        if (c.tid == 0) {
            taken = atomicAdd(&c.hdr->next_tile[0], 1u);
        }
        const uint4 v = warp_fold_pairs<false>(q, ft, c.lane);
        uint32_t next;
        if (!row_handoff(h, j, v, taken, c, next)) {
            return c.total;
        }
        ++j;
        if (next >= c.total || (tile_class(c, next) >> 1) != LQ) {
            return next;
        }
        tile = next;
    }
}

// Power warp of the GHASH pass: E_K(J0), L*H and the basis of H^d while the
// rows run, then fold levels 4..8 (shared tables), the object's sum and, once
// its last tile is in, the verdict (auth_ok and the object's slot).
__device__ __forceinline__ void open_power_loop(const uint8_t* smem, const BatchArgs& a, const BatchCta& c,
                                                const Handoff& h, uint32_t tile)
{
    constexpr unsigned long long T = kHornerThreads;
    const uint4* t4 = reinterpret_cast<const uint4*>(smem + kOpenFold) + 4 * 512;
    for (uint32_t j = 0; tile < c.total; ++j) {
        const TileRec tr = c.rec[tile];
        const uint32_t cta = tr.cta & kTileIndexMask;
        Slot* slot = c.st + tr.item;
        const BatchItem* it = a.items + tr.item;
        const uint32_t J = slot->aux[0];
        const uint32_t G = slot->aux[1];
        const uint64_t P = it->plen;
        const unsigned long long d = static_cast<unsigned long long>(G - 1 - cta) * J * T + 2ull;
        uint4 ej0, lh;
        unsigned long long uhi, ulo;
        open_power(it->src, a.kt.aes_t, a.rk, P, d, a.kt.gh_pow2, c.lane, ej0, lh, uhi, ulo);
        uint4 v;
        uint32_t next;
        if (!power_take(h, j, c.lane, v, next)) {
            return;
        }
        const uint4 fold = power_fold(v, t4, c.lane);
        unsigned long long shi, slo;
        if (batch_object_sum(slot, G, fold, uhi, ulo, c.lane, shi, slo) && c.lane == 0) {
            const int ok = open_verdict(it->src, P, shi, slo, lh, ej0);
            *it->auth_ok = ok;
            slot->aux[2] = static_cast<unsigned int>(ok);
        }
        tile = next;
    }
}

__global__ void __launch_bounds__(kSealThreads, 1) open_ghash_batch_kernel(const BatchArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x;
    pdl_release();
    fill_gh_smem(smem + kOpenGh, a.kt.gh_pow2 + kOpenChainLog2 * 512);
    for (int i = tid; i < (kFoldLevels + 1) * 512; i += blockDim.x) {
        reinterpret_cast<uint4*>(smem + kOpenFold)[i] = __ldg(a.kt.gh_pow2 + i);
    }
    const Handoff h = handoff_at(smem, kOpenBatchHandoff, kOpenBatchSync);
    if (tid == 0) {
        handoff_init(h);
    }
    pdl_wait();  // the plan kernel's workspace
    auto* hdr = reinterpret_cast<BatchHeader*>(a.ws);
    const BatchCta c{hdr, reinterpret_cast<Slot*>(a.ws + batch_slots_offset()),
                     reinterpret_cast<const TileRec*>(a.ws + batch_tiles_offset(a.count)), hdr->total_tiles,
                     tid, tid & 31, tid >> 5};
    uint32_t tile = first_tile(h.first, c, 0);
    if (c.warp == kPowerWarp) {
        open_power_loop(smem, a, c, h, tile);
    } else {
        uint32_t j = 0;
        while (tile < c.total) {
            switch (tile_class(c, tile) >> 1) {  // the GHASH pass does not touch the plaintext side
            case 0: tile = open_ghash_class<0>(smem, a, c, h, tile, j); break;
            case 1: tile = open_ghash_class<1>(smem, a, c, h, tile, j); break;
            case 2: tile = open_ghash_class<2>(smem, a, c, h, tile, j); break;
            case 3: tile = open_ghash_class<3>(smem, a, c, h, tile, j); break;
            default: tile = open_ghash_class<4>(smem, a, c, h, tile, j); break;
            }
        }
    }
    handoff_failed(h, c);
}

// Gated CTR over the same tiles (rows of kCtrThreads = kHornerThreads
// blocks). Each tile reads its object's verdict, written by
// open_ghash_batch_kernel earlier on the stream: authentic -> decrypt,
// otherwise zero the tile's plaintext bytes. Thread 0 takes the next index
// after this tile's rows (a CTA that reserved tiles ahead would hold them
// while other CTAs sit idle); it goes through a two-entry shared buffer so
// one barrier per tile suffices.
template <int LQ, bool PT>
__device__ __forceinline__ uint32_t ctr_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c, uint32_t tile,
                                              int cls, uint32_t& round)
{
    static_assert(kCtrThreads == kHornerThreads, "CTR tiles reuse the GHASH tile rows");
    constexpr int64_t T = kCtrThreads;
    volatile uint32_t* next_s = reinterpret_cast<volatile uint32_t*>(smem + kCtrBatchMisc);
    for (;; ++round) {
        const TileRec tr = c.rec[tile];
        const uint32_t cta = tr.cta & kTileIndexMask;
        const BatchItem* it = a.items + tr.item;
        const Slot& slot = c.st[tr.item];
        const uint32_t J = slot.aux[0];
        const uint32_t G = slot.aux[1];
        const int ok = static_cast<int>(slot.aux[2]);
        const uint64_t P = it->plen;
        const int64_t n = static_cast<int64_t>(P / 16u + ((P & 15u) != 0));
        const int64_t span = static_cast<int64_t>(J) * T;
        const uint8_t* frame = it->src;
        int lq;
        uint32_t load_r;
        load_class(frame + 13, lq, load_r);  // lq == LQ for this class
        (void)lq;
        CtrTile t{frame, it->capacity, it->dst, P, n - static_cast<int64_t>(G - cta) * span,
                  static_cast<int64_t>(J), {0u, 0u, 0u}, load_r};
        if (!ok) {
            ctr_zero_rows<PT>(t, c.tid);
        } else {
            const uint4 iv = load_bytes(frame + 1, 12);
            t.s012[0] = iv.x ^ a.rk[0];
            t.s012[1] = iv.y ^ a.rk[1];
            t.s012[2] = iv.z ^ a.rk[2];
            ctr_rows<LQ, PT>(t, a.rk, c.tid, c.lane);
        }
        if (c.tid == 0) {
            next_s[round & 1] = atomicAdd(&c.hdr->next_tile[1], 1u);
        }
        __syncthreads();
        const uint32_t next = next_s[round & 1];
        if (next >= c.total || tile_class(c, next) != cls) {
            ++round;
            return next;
        }
        tile = next;
    }
}

__global__ void __launch_bounds__(kCtrThreads, 1) open_ctr_batch_kernel(const BatchArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int tid = threadIdx.x;
    pdl_release();
    fill_aes_smem(smem, a.kt.aes_t);
    small_fill_open_tables(smem, a.kt.gh_pow2);
    pdl_wait();  // the verdicts of the GHASH pass
    auto* hdr = reinterpret_cast<BatchHeader*>(a.ws);
    const BatchCta c{hdr, reinterpret_cast<Slot*>(a.ws + batch_slots_offset()),
                     reinterpret_cast<const TileRec*>(a.ws + batch_tiles_offset(a.count)), hdr->total_tiles,
                     tid, tid & 31, tid >> 5};
    uint32_t tile = first_tile(reinterpret_cast<volatile uint32_t*>(smem + kCtrBatchMisc) + 2, c, 1);
    uint32_t round = 0;  // parity of the shared buffer entry, continued across classes
    while (tile < c.total) {
        const int cls = tile_class(c, tile);
        switch (cls) {
        case 0: tile = ctr_class<0, false>(smem, a, c, tile, cls, round); break;
        case 1: tile = ctr_class<0, true>(smem, a, c, tile, cls, round); break;
        case 2: tile = ctr_class<1, false>(smem, a, c, tile, cls, round); break;
        case 3: tile = ctr_class<1, true>(smem, a, c, tile, cls, round); break;
        case 4: tile = ctr_class<2, false>(smem, a, c, tile, cls, round); break;
        case 5: tile = ctr_class<2, true>(smem, a, c, tile, cls, round); break;
        case 6: tile = ctr_class<3, false>(smem, a, c, tile, cls, round); break;
        case 7: tile = ctr_class<3, true>(smem, a, c, tile, cls, round); break;
        case 8: tile = ctr_class<4, false>(smem, a, c, tile, cls, round); break;
        default: tile = ctr_class<4, true>(smem, a, c, tile, cls, round); break;
        }
    }

    // Small objects: one warp opens a whole object (GHASH, tag check, CTR),
    // so its plaintext waits for nothing outside the warp.
    const uint32_t small_count = hdr->small_count;
    const uint32_t* small_list = reinterpret_cast<const uint32_t*>(a.ws + batch_small_offset(a.count));
    for (;;) {
        uint32_t k = 0;
        if (c.lane == 0) {
            k = atomicAdd(&hdr->small_next[1], 1u);
        }
        k = __shfl_sync(0xffffffffu, k, 0);
        if (k >= small_count) {
            break;
        }
        open_object_warp(a.items + small_list[k], a.rk, a.kt.gh_pow2, smem, c.lane);
    }
}

}  // namespace dev
}  // namespace confkv
