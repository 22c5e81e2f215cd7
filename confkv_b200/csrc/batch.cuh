// Batched seal / open: one plan launch and one (seal) or two (open)
// persistent launches for any number of objects of any sizes and alignments.
//
// Objects of more than kSmallMaxBlocks blocks ("tile objects"; mid objects
// of up to kWarpMaxBlocks blocks only when the batch has too few of them for
// the warp path) are cut into rows of kHornerThreads blocks, aligned to the
// object's end (only row 0 can start before block 0). The batch's rows form one row space, tile objects
// back to back, which is cut into M chunks of equal estimated cost (rows
// plus a fixed charge per tile object). As in stream-K, a chunk may end
// inside one object and start inside another, so every SM gets the same
// work whatever the object sizes. The part of one object inside one chunk
// is a segment; it is processed like a tile (tiles.cuh) and its GHASH share
// is combined through the object's slot, the last segment writing the tag
// or verdict.
//
//   batch_plan_kernel    one CTA: validates every descriptor (status), puts
//                        small objects into size-bucket lists, routes the
//                        mid objects to warps or to rows, lays out the
//                        row space (tile objects grouped by alignment
//                        class), picks M, counts each object's segments and
//                        records each chunk's first row and tile object.
//   seal_batch_kernel    one CTA per SM; each takes chunks from a queue
//   open_ghash_batch_    (atomic head) and walks their segments. No CTA waits
//   kernel               for another. After the chunks, small objects, one
//   open_ctr_batch_      warp each (seal, open-CTR).
//   kernel
//
// Device-written workspace (caller-owned, any contents on entry):
//   [0, 256)            BatchHeader
//   [256, ...)          one Slot per object: acc, ticket, aux = {rows, segments, verdict}
//   [objs_offset, ...)  TileObj per tile object, then a sentinel
//   [chunks_offset, ...) ChunkRec per chunk (first row, first tile object), then a sentinel
//   [small_offset, ...) small objects (item indices): kSmallBuckets regions of
//                       `count` entries, one per size bucket
#pragma once

#include <cstddef>

#include "small.cuh"
#include "tiles.cuh"

namespace confkv {
namespace dev {

constexpr int kBatchMaxSms = 256;     // SMs the plan spreads chunks over
constexpr int kChunksPerSm = 4;       // chunks per SM for batches of many tile objects
constexpr int kChunksPerSmFew = 1;    // chunks per SM otherwise
constexpr uint32_t kMinChunkRows = 64;  // fewer chunks per SM while chunks would be shorter than this
constexpr uint32_t kMaxChunks = static_cast<uint32_t>(kChunksPerSm * kBatchMaxSms);
constexpr uint32_t kBatchMaxItems = 1u << 20;
constexpr int kPlanThreads = 1024;
constexpr uint64_t kBatchMaxBlocks = 0xfffffffeull;
constexpr uint32_t kCtrBatchMisc = kSmallSmem;      // after the small-object tables
constexpr uint32_t kCtrBatchSmem = kCtrBatchMisc + 64;
static_assert(kCtrBatchSmem + kSmemGapToday <= kSmemOptInLimit, "batched CTR shared memory exceeds the per-block limit");
// Small objects are handed out largest first, by size bucket: n <= 128,
// <= 256, <= 512, <= 1024 blocks (up to 2, 4, 8, 16 KiB), and bucket 4 for
// the mid objects (1025 .. kWarpMaxBlocks blocks, up to 32 KiB) when they take
// the warp path. Each bucket has its own list region of `count` entries,
// filled in the plan's first pass.
constexpr int kSmallBuckets = 5;
// Mid objects take one warp each when the batch's N warp-path objects
// (small + mid) are enough for the warps to beat the tile path:
//   N (rows_avg + o) 512 >= alpha max_n sms,
// rows_avg + o being a mid object's mean cost as a tile object (rows plus
// the segment charge) and max_n its largest size in blocks. A warp's
// throughput is about fixed, so warp-path throughput grows with N; a tile
// object's cost grows with its rows plus o, a warp's time with n. alpha
// comes from measured crossovers on B200 (32 KiB objects: seal at 11.5, open
// at 8.4 objects per SM; 20 KiB: about 8 and under 7): 2048 objects of
// 32 KiB ran 298 / 313 GB/s (seal / open) as warps against 249 / 200 as
// tiles, 1480 of them 218 / 238 against 254 / 201. With fewer objects, one
// warp's serial rows (up to 64) would end the call late, and they stay tile
// objects like the larger ones.
constexpr uint32_t kMidAlphaSeal = 26;
constexpr uint32_t kMidAlphaOpen = 19;
constexpr uint32_t kMidFlag = 0x80000000u;  // aux[0] of a mid object until the plan routes it

// Hand-off from the row warps to the power warp (two-stage fold, tiles.cuh):
// two buffers of 32 partials, and per buffer a FULL mbarrier (the 16 row
// warps arrived) and an EMPTY one (the power warp took the values).
constexpr uint32_t kHandoffBytes = 2 * 32 * 16;
constexpr uint32_t kHandoffSyncBytes = 96;   // mbarriers, queue words, the CTA context, the wait limit
constexpr uint32_t kWalkBytes = (kHornerThreads / 32) * 16;  // one WalkSlot per row warp
// Batched seal shared memory: AES tables, the chain table H^512 (H^32 for
// small objects), the row-warp fold tables H^8, H^1, H^2, H^4 (the slots the
// small-object path reads), the hand-off buffers and their mbarriers.
constexpr uint32_t kSealBatchFold = kAesBytes + kGhBytes;
constexpr uint32_t kSealBatchHandoff = kSealBatchFold + 4 * 8192u;
constexpr uint32_t kSealBatchSync = kSealBatchHandoff + kHandoffBytes;
constexpr uint32_t kSealBatchWalk = kSealBatchSync + kHandoffSyncBytes;
constexpr uint32_t kSealBatchSmem = kSealBatchWalk + kWalkBytes;
static_assert(kSealBatchFold == kSmallFold, "the small-object path reads the seal fold slots");
static_assert(kSealBatchSmem + kSmemGapToday <= kSmemOptInLimit, "batched seal shared memory exceeds the per-block limit");
// Shared memory of the batched GHASH passes (open, two-pass seal): the
// replicated table of the chain multiplier (kGhW-bit windows when
// kGhashTable5: 26 (W = 5) or 22 (W = 6) lookups of 16 B per multiply
// instead of 32, i.e. 3.25 or 2.75 shared-memory wavefronts per block
// instead of 4), the fold tables of H^1 .. H^8 (row warps) and, when room is
// left, of H^16 .. H^256 (the power warp reads them from global memory
// otherwise: the 176 KiB of a 6-bit table leave none), the compact table of
// H^512 (the chain combine), the hand-off.
constexpr bool kGhashTable5 = true;
constexpr int kGhPassFoldLevels = (kGhashTable5 && kGhW > 5) ? 4 : kFoldLevels;
constexpr uint32_t kGhPassGh = 0;
constexpr uint32_t kGhPassFold = kGhPassGh + (kGhashTable5 ? static_cast<uint32_t>(kGh5RepBytes) : kGhBytes);
constexpr uint32_t kGhPassHt = kGhPassFold + static_cast<uint32_t>(kGhPassFoldLevels) * 8192u;
constexpr uint32_t kOpenBatchHandoff = kGhPassHt + 8192u;
constexpr uint32_t kOpenBatchSync = kOpenBatchHandoff + kHandoffBytes;
constexpr uint32_t kOpenBatchWalk = kOpenBatchSync + kHandoffSyncBytes;
constexpr uint32_t kOpenBatchSmem = kOpenBatchWalk + kWalkBytes;
static_assert(kOpenBatchSmem + kSmemGapToday <= kSmemOptInLimit, "batched GHASH shared memory exceeds the per-block limit");

// Alignment classes: 2 v + p, v = the frame's ciphertext class (seal: store
// funnel word part 0..3, 4 = aligned; open: load funnel word part, same
// coding) and p = 1 when the plaintext side (seal src, open dst) is 16-B
// aligned. Each tile object carries its class; the work kernels run a loop
// specialised for it and switch loops only when the class changes.
constexpr int kClasses = 10;

struct BatchHeader {
    unsigned long long total_rows;  // R: rows of all tile objects
    uint32_t chunks;                // M (0 when there are no tile objects)
    uint32_t next_chunk[2];         // queue heads: [0] seal / open GHASH, [1] open CTR
    uint32_t tile_objects;          // K
    uint32_t small_count;           // warp-path objects (small, and mid when routed), one warp each
    uint32_t fault;                 // nonzero: a work kernel's hand-off wait gave up (results invalid)
    uint32_t small_next[2];         // small-object queue heads: [0] seal, [1] open
    uint32_t small_bucket[5];       // objects per small-object bucket (kSmallBuckets)
    uint32_t seal_two_pass;         // seal: 1 = CTR pass, then GHASH pass (seal_two_pass_wins); 0 = one fused pass
};
static_assert(sizeof(BatchHeader) <= 256, "batch header fits its 256-byte area");

// A tile object in the row space: its first row, descriptor index, rows and
// alignment class.
struct TileObj {
    unsigned long long row_start;
    uint32_t item;
    uint32_t meta;                  // rows (bits 0-23) | class << 24
};
constexpr uint32_t kRowsMask = 0x00ffffffu;
static_assert((kBatchMaxBlocks + kHornerThreads - 1) / kHornerThreads <= kRowsMask, "rows fit the meta field");

__host__ __device__ constexpr size_t batch_round256(size_t x) { return (x + 255) / 256 * 256; }
__host__ __device__ constexpr size_t batch_slots_offset() { return 256; }
__host__ __device__ constexpr size_t batch_objs_offset(size_t count)
{
    return 256 + batch_round256(count * sizeof(Slot));
}
__host__ __device__ constexpr size_t batch_chunks_offset(size_t count)
{
    return batch_objs_offset(count) + batch_round256((count + 1) * sizeof(TileObj));
}
// Planned per-segment overhead, in rows of the seal loop: a segment's fold,
// hand-off, descriptor fetch and pipeline start cost about three rows on
// B200, so chunks of many small objects get fewer rows.
constexpr uint32_t kSegmentCostRows = 5;

// A chunk of the row space: its first row and the tile object holding it.
struct ChunkRec {
    unsigned long long row_start;
    uint32_t first;
    uint32_t pad;
};

__host__ __device__ constexpr size_t batch_small_offset(size_t count)
{
    return batch_chunks_offset(count) + (kMaxChunks + 1) * sizeof(ChunkRec);
}
__host__ __device__ constexpr size_t batch_workspace_bytes(size_t count)
{
    return batch_small_offset(count) + kSmallBuckets * count * sizeof(uint32_t);
}

// First row of chunk c and the chunk holding row x (0 <= x < R), for M
// chunks of R rows: chunk c = [floor(c R / M), floor((c+1) R / M)).
__host__ __device__ __forceinline__ unsigned long long chunk_row(uint32_t c, unsigned long long R, uint32_t M)
{
    return static_cast<unsigned long long>(c) * R / M;
}
__host__ __device__ __forceinline__ uint32_t chunk_of(unsigned long long x, unsigned long long R, uint32_t M)
{
    return static_cast<uint32_t>(((x + 1) * M - 1) / R);
}

// Chunks for R rows of K tile objects on `sms` SMs. With at least
// kChunksPerSm tile objects per SM of mixed sizes the per-object cost
// estimate is least exact and more chunks let the queue even out the SMs:
// kChunksPerSm per SM; otherwise kChunksPerSmFew, since every chunk boundary
// inside an object adds a segment (fold, hand-off, pipeline restart): on
// B200 one chunk per SM ran batches of a few large objects 0.4-0.9 % faster
// than two, and two 0.8 % faster than four. A batch is `uniform` when its
// largest tile object has at most kUniformRowsRatio times the rows of its
// smallest: equal chunks then already balance the SMs. Fewer while a chunk
// would be shorter than kMinChunkRows, at least one per SM, never more than R
// (so no chunk is empty).
constexpr uint32_t kUniformRowsRatio = 2;
__host__ __device__ __forceinline__ uint32_t batch_chunk_count(unsigned long long R, uint32_t K, uint32_t sms,
                                                              bool uniform)
{
    if (R == 0) {
        return 0;
    }
    const unsigned long long cap =
        K >= static_cast<unsigned long long>(kChunksPerSm) * sms && !uniform ? kChunksPerSm : kChunksPerSmFew;
    unsigned long long per = R / (static_cast<unsigned long long>(sms) * kMinChunkRows);
    per = per < 1 ? 1 : (per > cap ? cap : per);
    const unsigned long long m = per * sms;
    return static_cast<uint32_t>(m < R ? m : R);
}

// The batched seal runs in one of two ways. Fused: seal_batch_kernel's row
// warps encrypt and hash each segment in one pass (AES and GHASH tables share
// the shared-memory pipe). Two passes: seal_batch_kernel only encrypts, then
// seal_ghash_batch_kernel reads the ciphertext back and hashes it on four
// chains, one of them on the integer pipes (the batched open's GHASH pass),
// which leaves the shared-memory pipe less loaded per block. Every segment
// then pays its start-up and fold twice, and the second pass its own launch
// tail, so two passes win only on batches with many rows per SM and long
// tile objects (a row is kHornerThreads blocks, 8 KiB). Measured on B200
// with the 6-bit-window GHASH pass (seal GB/s, fused -> two passes; rows per
// SM, rows per object): 4 x 64 MiB 470 -> 518 (221, 8192); 8 x 32 MiB
// 470 -> 506 (221, 4096); 64 x 2 MiB 436 -> 444 (110, 256); 128 x 1 MiB 429 -> 439 (110, 128); 192 x 768 KiB
// 435 -> 438 (125, 96); 96 x 2 MiB 452 -> 477 (166, 256); ties at 112 x
// 1 MiB 423 / 423 (97, 128), 56 x 2 MiB (97, 256) and 256 x 512 KiB (110,
// 64); fused wins at 96 x 1 MiB 412 -> 409 (83), 80 x 1 MiB 405 -> 389 (69),
// 64 x 1 MiB 385 -> 370 (55), 384 x 384 KiB 421 -> 417 (125, 48), 512 x
// 256 KiB 405 -> 388 (110, 32), 1024 x 128 KiB 375 -> 338 (110, 16) and the
// 4096-object ragged batch (~23 rows per tile object) 374 -> 355.
constexpr unsigned long long kTwoPassMinRowsPerSm = 104;
constexpr unsigned long long kTwoPassMinRowsPerObject = 96;

__host__ __device__ __forceinline__ bool seal_two_pass_wins(unsigned long long R, uint32_t K, uint32_t sms)
{
    return K != 0 && R >= kTwoPassMinRowsPerSm * sms && R >= kTwoPassMinRowsPerObject * K;
}

struct BatchArgs {
    BatchItem* items;
    uint8_t* ws;
    uint32_t count;
    // Test-only stall injection (host switch CONFKV_B200_TEST_HANDOFF_STALL):
    // nonzero makes the seal power warp stop taking hand-offs, so the row
    // warps' bounded waits run out after wait_ns and the batch reports a
    // fault. wait_ns is kWaitLimitNs otherwise.
    uint32_t stall;
    unsigned long long wait_ns;
    uint32_t rk[44];
    KeyTables kt;
    ClmulConst open_cm;  // the batched GHASH passes' chain multiplier for their integer-pipe chains
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

// ------------------------------------------------------------------ plan

// Block-wide exclusive scan of one 64-bit value per thread (kPlanThreads
// threads, all calling); `warp_sums` holds kPlanThreads / 32 values. Returns
// the thread's exclusive prefix; *total gets the sum.
__device__ __forceinline__ unsigned long long plan_scan(unsigned long long v, unsigned long long* warp_sums,
                                                        unsigned long long* total)
{
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    unsigned long long incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const unsigned long long u = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) {
            incl += u;
        }
    }
    if (lane == 31) {
        warp_sums[warp] = incl;
    }
    __syncthreads();
    if (warp == 0) {
        unsigned long long w = warp_sums[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const unsigned long long u = __shfl_up_sync(0xffffffffu, w, d);
            if (lane >= d) {
                w += u;
            }
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    *total = warp_sums[kPlanThreads / 32 - 1];
    const unsigned long long before = warp > 0 ? warp_sums[warp - 1] : 0ull;
    __syncthreads();  // warp_sums may be reused
    return before + incl - v;
}

// Block-wide inclusive prefix maximum of one value per thread (kPlanThreads
// threads, all calling); `warp_max` holds kPlanThreads / 32 values.
__device__ __forceinline__ uint32_t plan_scan_max(uint32_t v, uint32_t* warp_max)
{
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) {
            v = u > v ? u : v;
        }
    }
    if (lane == 31) {
        warp_max[warp] = v;
    }
    __syncthreads();
    if (warp == 0) {
        uint32_t w = warp_max[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t u = __shfl_up_sync(0xffffffffu, w, d);
            if (lane >= d) {
                w = u > w ? u : w;
            }
        }
        warp_max[lane] = w;
    }
    __syncthreads();
    const uint32_t before = warp > 0 ? warp_max[warp - 1] : 0u;
    return before > v ? before : v;
}

// `open` selects the descriptor rules: seal needs capacity >= P + 29; open
// needs frame length >= P + 29 and an auth_ok pointer. sms = SMs the work
// kernels run on (at most kBatchMaxSms). The row space holds the tile
// objects grouped by alignment class (so a CTA's segments mostly share one
// specialised loop); the order inside a class follows the atomics.
__global__ void __launch_bounds__(kPlanThreads) batch_plan_kernel(BatchItem* items, uint32_t count,
                                                                  uint8_t* ws, int open, uint32_t sms)
{
    __shared__ unsigned long long warp_sums[kPlanThreads / 32];
    __shared__ unsigned long long class_rows[kClasses];
    __shared__ unsigned int class_objs[kClasses];
    __shared__ unsigned int class_cursor[kClasses];
    __shared__ unsigned long long mid_rows[kClasses];
    __shared__ unsigned int mid_objs[kClasses];
    __shared__ uint32_t route_mid;
    __shared__ unsigned int mid_max_n;
    __shared__ unsigned int tile_min_rows;  // over the tile and mid objects
    __shared__ unsigned int tile_max_rows;
    __shared__ unsigned long long total_rows_s;
    __shared__ uint32_t tile_objs_s;
    __shared__ uint32_t chunks_s;
    __shared__ unsigned int small_fill[kSmallBuckets];
    __shared__ uint32_t chunk_mark[kPlanThreads];
    __shared__ uint32_t warp_marks[kPlanThreads / 32];
    static_assert(kMaxChunks <= kPlanThreads, "one plan thread per chunk");
    BatchHeader* hdr = reinterpret_cast<BatchHeader*>(ws);
    Slot* st = reinterpret_cast<Slot*>(ws + batch_slots_offset());
    TileObj* objs = reinterpret_cast<TileObj*>(ws + batch_objs_offset(count));
    ChunkRec* chunks = reinterpret_cast<ChunkRec*>(ws + batch_chunks_offset(count));
    uint32_t* small_list = reinterpret_cast<uint32_t*>(ws + batch_small_offset(count));
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    constexpr uint64_t T = kHornerThreads;
    pdl_release();
    if (tid < kSmallBuckets) {
        small_fill[tid] = 0;
    }
    if (tid < kClasses) {
        class_rows[tid] = 0;
        class_objs[tid] = 0;
        mid_rows[tid] = 0;
        mid_objs[tid] = 0;
    }
    if (tid == 0) {
        mid_max_n = 0;
        tile_min_rows = 0xffffffffu;
        tile_max_rows = 0;
    }
    chunk_mark[tid] = 0;
    __syncthreads();
    pdl_wait();  // descriptors and workspace may belong to earlier work on the stream

    // Pass 1: validate, rows per tile object (small and invalid objects have
    // none), reset the slot (aux[1] keeps the class until pass 3), the
    // per-class totals, and the small objects into their bucket's list (one
    // shared atomic per class or bucket present in a warp).
    static_assert(offsetof(BatchItem, dst) == 8 && offsetof(BatchItem, plen) == 16 &&
                      offsetof(BatchItem, capacity) == 24 && offsetof(BatchItem, auth_ok) == 32,
                  "pass 1 decodes the descriptor's first 48 bytes");
    // The fields pass 1 reads (the first 48 bytes of a descriptor) are
    // loaded one iteration ahead, so the loop pays one memory latency in all
    // rather than one per iteration.
    auto fetch = [&](uint32_t i, uint4 (&d)[3]) {
        if (i < count) {
            const uint4* q = reinterpret_cast<const uint4*>(items + i);
            d[0] = q[0];
            d[1] = q[1];
            d[2] = q[2];
        }
    };
    uint4 cur[3];
    fetch(static_cast<uint32_t>(tid), cur);
    for (uint32_t base = 0; base < count; base += kPlanThreads) {
        const uint32_t i = base + static_cast<uint32_t>(tid);
        uint4 nxt[3];
        fetch(i + kPlanThreads, nxt);
        int key = -1;   // alignment class of a tile object
        int mkey = -1;  // alignment class of a mid object
        int skey = -1;  // size bucket of a small or mid object
        uint32_t rows = 0;
        uint32_t mid_n = 0;
        if (i < count) {
            // {src, dst}, {plen, capacity}, {auth_ok, iv[0..1]}
            const uint8_t* src = reinterpret_cast<const uint8_t*>(
                (static_cast<unsigned long long>(cur[0].y) << 32) | cur[0].x);
            const uint8_t* dst = reinterpret_cast<const uint8_t*>(
                (static_cast<unsigned long long>(cur[0].w) << 32) | cur[0].z);
            const uint64_t P = (static_cast<uint64_t>(cur[1].y) << 32) | cur[1].x;
            const uint64_t capacity = (static_cast<uint64_t>(cur[1].w) << 32) | cur[1].z;
            const bool has_auth = (cur[2].x | cur[2].y) != 0u;
            const uint64_t n = P / 16u + ((P & 15u) != 0);
            bool ok = src != nullptr && dst != nullptr && n <= kBatchMaxBlocks && capacity >= P + 29u;
            if (open) {
                ok = ok && has_auth;
            }
            const bool small = ok && n <= kSmallMaxBlocks;
            rows = ok && !small ? static_cast<uint32_t>((n + T - 1) / T) : 0u;
            items[i].status = ok ? 0 : -1;
            if (open && !ok && has_auth) {
                // a rejected open never leaves an earlier call's verdict behind
                *reinterpret_cast<int*>((static_cast<unsigned long long>(cur[2].y) << 32) | cur[2].x) = 0;
            }
            if (rows != 0) {
                int v;
                uint32_t r;
                if (open) {
                    load_class(src + 13, v, r);
                    key = 2 * v + ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
                } else {
                    store_class(dst + 13, v, r);
                    key = 2 * v + ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
                }
            }
            const bool mid = rows != 0 && n <= kWarpMaxBlocks;
            if (small) {
                skey = n <= 128 ? 0 : (n <= 256 ? 1 : (n <= 512 ? 2 : 3));
            } else if (mid) {
                // listed for the warp path and counted apart until the plan
                // knows how many warp-path objects there are
                skey = 4;
                mkey = key;
                key = -1;
                mid_n = static_cast<uint32_t>(n);
            }
            Slot& s = st[i];
            s.acc_hi = 0;
            s.acc_lo = 0;
            s.ticket = 0;
            s.aux[0] = mid ? (rows | kMidFlag) : rows;
            s.aux[1] = static_cast<uint32_t>(mid ? mkey : key);
            s.aux[2] = 0;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const unsigned sum = __reduce_add_sync(peers, key >= 0 ? rows : 0u);  // at most 32 x 2^23
        if (key >= 0 && lane == __ffs(peers) - 1) {
            atomicAdd(&class_rows[key], static_cast<unsigned long long>(sum));
            atomicAdd(&class_objs[key], static_cast<unsigned>(__popc(peers)));
        }
        const unsigned warp_max_n = __reduce_max_sync(0xffffffffu, mid_n);
        if (lane == 0 && warp_max_n != 0) {
            atomicMax(&mid_max_n, warp_max_n);
        }
        const unsigned warp_min_rows = __reduce_min_sync(0xffffffffu, rows != 0 ? rows : 0xffffffffu);
        const unsigned warp_max_rows = __reduce_max_sync(0xffffffffu, rows);
        if (lane == 0 && warp_max_rows != 0) {
            atomicMin(&tile_min_rows, warp_min_rows);
            atomicMax(&tile_max_rows, warp_max_rows);
        }
        const unsigned mpeers = __match_any_sync(0xffffffffu, mkey);
        const unsigned msum = __reduce_add_sync(mpeers, mkey >= 0 ? rows : 0u);
        if (mkey >= 0 && lane == __ffs(mpeers) - 1) {
            atomicAdd(&mid_rows[mkey], static_cast<unsigned long long>(msum));
            atomicAdd(&mid_objs[mkey], static_cast<unsigned>(__popc(mpeers)));
        }
        const unsigned speers = __match_any_sync(0xffffffffu, skey);
        if (skey >= 0) {
            const int leader = __ffs(speers) - 1;
            unsigned pos = 0;
            if (lane == leader) {
                pos = atomicAdd(&small_fill[skey], static_cast<unsigned>(__popc(speers)));
            }
            pos = __shfl_sync(speers, pos, leader) + static_cast<unsigned>(__popc(speers & ((1u << lane) - 1u)));
            small_list[static_cast<size_t>(skey) * count + pos] = i;
        }
#pragma unroll
        for (int w = 0; w < 3; ++w) {
            cur[w] = nxt[w];
        }
    }
    __syncthreads();
    if (tid == 0) {
        // mid objects take the warp path when there are enough warp-path
        // objects to beat their cost as tile objects
        unsigned long long warp_objs = 0;
        for (int b = 0; b < kSmallBuckets; ++b) {
            warp_objs += small_fill[b];
        }
        unsigned long long mid_cost = 0;  // sum of (rows + o) over mid objects
        for (int c = 0; c < kClasses; ++c) {
            mid_cost += mid_rows[c] + static_cast<unsigned long long>(kSegmentCostRows) * mid_objs[c];
        }
        const unsigned long long mids = small_fill[4];
        const unsigned long long alpha = open ? kMidAlphaOpen : kMidAlphaSeal;
        const uint32_t route =
            mids != 0 && warp_objs * mid_cost * kHornerThreads >= alpha * mid_max_n * sms * mids ? 1u : 0u;
        route_mid = route;
        unsigned long long R = 0;
        uint32_t K = 0;
        for (int c = 0; c < kClasses; ++c) {
            class_cursor[c] = K;
            K += class_objs[c] + (route ? 0u : mid_objs[c]);
            R += class_rows[c] + (route ? 0ull : mid_rows[c]);
        }
        const bool uniform =
            K != 0 && static_cast<unsigned long long>(tile_max_rows) <=
                          static_cast<unsigned long long>(kUniformRowsRatio) * tile_min_rows;
        const uint32_t M = batch_chunk_count(R, K, sms, uniform);
        total_rows_s = R;
        tile_objs_s = K;
        chunks_s = M;
        hdr->total_rows = R;
        hdr->chunks = M;
        hdr->next_chunk[0] = 0;
        hdr->next_chunk[1] = 0;
        hdr->tile_objects = K;
        hdr->fault = 0;
        hdr->seal_two_pass = !open && seal_two_pass_wins(R, K, sms) ? 1u : 0u;
        objs[K] = TileObj{R, 0xffffffffu, 0u};
    }
    __syncthreads();
    if (tid == 32) {
        unsigned int total = 0;
        for (int b = 0; b < kSmallBuckets; ++b) {
            const unsigned int nb = b == 4 && !route_mid ? 0u : small_fill[b];
            hdr->small_bucket[b] = nb;
            total += nb;
        }
        hdr->small_count = total;
        hdr->small_next[0] = 0;
        hdr->small_next[1] = 0;
    }
    if (tile_objs_s == 0) {
        return;  // small objects only: nothing to place
    }

    // Pass 2: place the tile objects, class by class (each slot's rows and
    // class loaded one iteration ahead, as in pass 1).
    auto fetch_slot = [&](uint32_t i, uint32_t& rows, uint32_t& cls) {
        if (i < count) {
            rows = st[i].aux[0];
            cls = st[i].aux[1];
        }
    };
    uint32_t cur_rows = 0, cur_cls = 0;
    fetch_slot(static_cast<uint32_t>(tid), cur_rows, cur_cls);
    for (uint32_t base = 0; base < count; base += kPlanThreads) {
        const uint32_t i = base + static_cast<uint32_t>(tid);
        uint32_t next_rows = 0, next_cls = 0;
        fetch_slot(i + kPlanThreads, next_rows, next_cls);
        int key = -1;
        uint32_t rows = 0;
        if (i < count) {
            rows = cur_rows & ~kMidFlag;
            if ((cur_rows & kMidFlag) != 0u) {
                // a mid object: a tile object unless it took the warp path
                if (route_mid) {
                    rows = 0;
                } else {
                    st[i].aux[0] = rows;
                }
            }
            if (rows != 0) {
                key = static_cast<int>(cur_cls);
            }
        }
        cur_rows = next_rows;
        cur_cls = next_cls;
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        if (key >= 0) {
            const int leader = __ffs(peers) - 1;
            unsigned pos = 0;
            if (lane == leader) {
                pos = atomicAdd(&class_cursor[key], static_cast<unsigned>(__popc(peers)));
            }
            pos = __shfl_sync(peers, pos, leader) + static_cast<unsigned>(__popc(peers & ((1u << lane) - 1u)));
            objs[pos].item = i;
            objs[pos].meta = rows | (static_cast<uint32_t>(key) << 24);
        }
    }
    __syncthreads();

    // Pass 3: row starts (a scan over contiguous ranges of the placed
    // objects), each object's segment count, the tile object holding each
    // chunk's first row.
    const unsigned long long R = total_rows_s;
    const uint32_t K = tile_objs_s;
    const uint32_t M = chunks_s;
    const uint32_t per = (K + kPlanThreads - 1) / kPlanThreads;
    const uint32_t lo = static_cast<uint32_t>(tid) * per < K ? static_cast<uint32_t>(tid) * per : K;
    const uint32_t hi = lo + per < K ? lo + per : K;
    unsigned long long mine = 0;
    for (uint32_t k = lo; k < hi; ++k) {
        mine += objs[k].meta & kRowsMask;
    }
    unsigned long long total;
    unsigned long long row = plan_scan(mine, warp_sums, &total);
    // Chunks are cut in a cost space where tile object k weighs its rows
    // plus o (kSegmentCostRows): object k covers costs [P_k, P_k + o + rows)
    // with P_k = S_k + o k, its overhead first. Chunk c starts at cost
    // x_c = floor(c C / M), C = R + o K, which maps to row
    // S_k + max(0, x_c - P_k - o) of the object holding x_c; row r of object k
    // (cost y = P_k + o + r - S_k) lies in chunk chunk_of(y, C, M). Narrow
    // chunks (under 2 (o + 1) cost units) drop the overhead weight (o = 0,
    // equal rows), so no chunk is empty.
    const unsigned long long o_full = kSegmentCostRows;
    const unsigned long long C_full = R + o_full * K;
    const unsigned long long o = M != 0 && C_full / M >= 2 * (o_full + 1) ? o_full : 0ull;
    const unsigned long long C = R + o * K;
    // x_c = c q + floor(c r / M) with q = C / M, r = C mod M (c r < 2^20:
    // a 32-bit division), so the per-chunk work needs no 64-bit division.
    const unsigned long long q = M != 0 ? C / M : 0ull;
    const uint32_t r = M != 0 ? static_cast<uint32_t>(C - q * M) : 0u;
    auto chunk_cost = [&](uint32_t c) { return c * q + (c * r) / M; };
    for (uint32_t k = lo; k < hi; ++k) {
        const uint32_t rows = objs[k].meta & kRowsMask;
        objs[k].row_start = row;
        const unsigned long long p = row + o * k;  // P_k
        const uint32_t first = chunk_of(p + o, C, M);
        const uint32_t last = chunk_of(p + o + rows - 1, C, M);
        st[objs[k].item].aux[1] = last - first + 1;
        // the first chunk whose first cost falls in [P_k, P_k + o + rows), if any
        uint32_t c = chunk_of(p, C, M);
        c = chunk_cost(c) == p ? c : c + 1;
        if (c <= last) {
            chunk_mark[c] = k + 1;
        }
        row += rows;
    }
    __syncthreads();
    // Chunk c's tile object: the last mark at or before c (a prefix max over
    // the chunks, one thread each); its first row follows from x_c.
    const uint32_t mark = static_cast<uint32_t>(tid) < M ? chunk_mark[tid] : 0u;
    const uint32_t owner = plan_scan_max(mark, warp_marks) - 1;
    if (static_cast<uint32_t>(tid) < M) {
        const uint32_t c = static_cast<uint32_t>(tid);
        const unsigned long long start = objs[owner].row_start;
        const unsigned long long p = start + o * owner;
        const unsigned long long x = chunk_cost(c);
        chunks[c] = ChunkRec{start + (x > p + o ? x - p - o : 0ull), owner, 0u};
    }
    if (tid == 0) {
        chunks[M] = ChunkRec{R, K, 0u};
    }
}

// Final GHASH sum of a segment's object: an object in one segment multiplies
// its fold by H^2 directly; otherwise each segment's share goes through the
// object's slot and only the last to arrive gets the sum. Power warp only;
// returns true where (shi, slo) holds the sum.
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

// Shared state of the work kernels. R, M and the workspace views sit in a
// shared-memory context block (kCtxBytes at `ctx`, written by thread 0, read
// where used through volatile loads), so that none of them is held in
// registers across a segment's rows.
constexpr uint32_t kCtxBytes = 40;
struct BatchCta {
    BatchHeader* hdr;        // the workspace (a kernel parameter)
    const uint8_t* ctx;
    int tid;
    int lane;
    int warp;
};

__device__ __forceinline__ unsigned long long ctx_u64(const BatchCta& c, int off)
{
    return *reinterpret_cast<const volatile unsigned long long*>(c.ctx + off);
}
__device__ __forceinline__ unsigned long long cta_rows(const BatchCta& c) { return ctx_u64(c, 0); }
__device__ __forceinline__ uint32_t cta_chunks(const BatchCta& c)
{
    return *reinterpret_cast<const volatile uint32_t*>(c.ctx + 8);
}
__device__ __forceinline__ const TileObj* cta_objs(const BatchCta& c)
{
    return reinterpret_cast<const TileObj*>(ctx_u64(c, 16));
}
__device__ __forceinline__ const ChunkRec* cta_chunk_recs(const BatchCta& c)
{
    return reinterpret_cast<const ChunkRec*>(ctx_u64(c, 24));
}
__device__ __forceinline__ Slot* cta_slots(const BatchCta& c)
{
    return reinterpret_cast<Slot*>(ctx_u64(c, 32));
}

// The caller's next barrier publishes thread 0's context writes.
__device__ __forceinline__ BatchCta batch_cta(const BatchArgs& a, uint8_t* ctx, int tid)
{
    auto* hdr = reinterpret_cast<BatchHeader*>(a.ws);
    if (tid == 0) {
        *reinterpret_cast<volatile unsigned long long*>(ctx) = hdr->total_rows;
        *reinterpret_cast<volatile uint32_t*>(ctx + 8) = hdr->chunks;
        *reinterpret_cast<volatile unsigned long long*>(ctx + 16) =
            reinterpret_cast<unsigned long long>(a.ws + batch_objs_offset(a.count));
        *reinterpret_cast<volatile unsigned long long*>(ctx + 24) =
            reinterpret_cast<unsigned long long>(a.ws + batch_chunks_offset(a.count));
        *reinterpret_cast<volatile unsigned long long*>(ctx + 32) =
            reinterpret_cast<unsigned long long>(a.ws + batch_slots_offset());
    }
    return BatchCta{hdr, ctx, tid, tid & 31, tid >> 5};
}

// Position in the row space: chunk `chunk`, tile object k. The rows left in
// the chunk start at max(first row of the chunk, first row of object k).
struct Cursor {
    uint32_t chunk;
    uint32_t k;
};

// Opens chunk `chunk`; false once the queue is exhausted.
__device__ __forceinline__ bool cursor_open(const BatchCta& c, uint32_t chunk, Cursor& cur)
{
    if (chunk >= cta_chunks(c)) {
        return false;
    }
    cur.chunk = chunk;
    cur.k = cta_chunk_recs(c)[chunk].first;
    return true;
}

// The segment at the cursor: rows [r0, r1) of tile object k, whose rows are
// [0, rows) (row r = blocks n - (rows - r) T .. + T); `last` when it ends
// the chunk.
struct Segment {
    uint32_t item;
    uint32_t rows;
    uint32_t r0;
    uint32_t r1;
    bool last;
};

__device__ __forceinline__ Segment segment_at(const BatchCta& c, const Cursor& cur)
{
    const TileObj o = cta_objs(c)[cur.k];
    const ChunkRec* cr = cta_chunk_recs(c) + cur.chunk;
    const unsigned long long a0 = cr[0].row_start;
    const unsigned long long b = cr[1].row_start;
    const uint32_t rows = o.meta & kRowsMask;
    const unsigned long long end = o.row_start + rows;
    const unsigned long long a = a0 > o.row_start ? a0 : o.row_start;
    return Segment{o.item, rows, static_cast<uint32_t>(a - o.row_start),
                   static_cast<uint32_t>((b < end ? b : end) - o.row_start), end >= b};
}

// Moves past segment sg; true when that ends the chunk (otherwise the next
// tile object starts where this one ends in the row space).
__device__ __forceinline__ bool cursor_step(Cursor& cur, const Segment& sg)
{
    if (sg.last) {
        return true;
    }
    ++cur.k;
    return false;
}

__device__ __forceinline__ int cursor_class(const BatchCta& c, const Cursor& cur)
{
    return static_cast<int>(cta_objs(c)[cur.k].meta >> 24);
}

// Row-warp walk state in shared memory, one slot per row warp: [0] chunk,
// [1] tile object of the next segment (kChunkEnd after a chunk's last one),
// [2] hand-off count. All lanes hold the same values, so every lane writes
// and reads its warp's slot, and none of it stays in registers across a
// segment's rows. The slot's address is rebuilt from the shared base where
// used.
constexpr uint32_t kChunkEnd = 0xffffffffu;
struct WalkSlot {
    uint8_t* base;   // shared base + the kernel's walk offset
};

__device__ __forceinline__ volatile uint32_t* walk_word(const WalkSlot& ws, int i)
{
    return reinterpret_cast<volatile uint32_t*>(ws.base + 16 * (threadIdx.x >> 5)) + i;
}
__device__ __forceinline__ Cursor walk_cursor(const WalkSlot& ws)
{
    return Cursor{*walk_word(ws, 0), *walk_word(ws, 1)};
}
// Opens `chunk` into the slot; false once the queue is exhausted.
__device__ __forceinline__ bool walk_open(const BatchCta& c, uint32_t chunk, const WalkSlot& ws)
{
    Cursor cur;
    if (!cursor_open(c, chunk, cur)) {
        return false;
    }
    *walk_word(ws, 0) = cur.chunk;
    *walk_word(ws, 1) = cur.k;
    return true;
}

// First block of segment sg (negative only when r0 = 0 and the object's first
// row is partial) and the power d of its GHASH share: (rows - r1) T blocks
// follow the segment, plus the length block.
__device__ __forceinline__ int64_t segment_base(const Segment& sg, uint64_t P)
{
    const int64_t n = static_cast<int64_t>(P / 16u + ((P & 15u) != 0));
    return n - static_cast<int64_t>(sg.rows - sg.r0) * kHornerThreads;
}
__device__ __forceinline__ unsigned long long segment_power(const Segment& sg)
{
    return static_cast<unsigned long long>(sg.rows - sg.r1) * kHornerThreads + 2ull;
}

// First chunk of this CTA (all threads); the barriers bracket the shared
// broadcast.
__device__ __forceinline__ uint32_t first_chunk(volatile uint32_t* next_s, const BatchCta& c, int pass)
{
    if (c.tid == 0) {
        *next_s = atomicAdd(&c.hdr->next_chunk[pass], 1u);
    }
    __syncthreads();
    const uint32_t t = *next_s;
    __syncthreads();
    return t;
}

// ------------------------------------------------------------- hand-off
//
// Seal and open-GHASH CTAs run their segments as a pipeline: the 16 row warps
// compute a segment's rows and the first fold stage, hand 32 values to the
// power warp and go on with the next segment, while the power warp finishes
// the fold, the object's sum and the tag (seal) or verdict (open). Hand-off
// j uses buffer j & 1; its FULL mbarrier completes when the 16 row warps
// arrived, its EMPTY mbarrier when the power warp has read the values, so a
// buffer is rewritten only after it was read. Both sides walk the same
// segments: at the end of a chunk thread 0 takes the next chunk index after
// its rows and passes it along with the values.

// Shared-memory views of the hand-off (kHandoffBytes of buffers at part_off,
// kHandoffSyncBytes of mbarriers and words at sync_off).
struct Handoff {
    uint4* part;               // [2][32] fold values V_p
    uint64_t* full;            // [2]
    uint64_t* empty;           // [2]
    volatile uint32_t* next;   // [2] chunk index taken after the buffer's segment (when it ended a chunk)
    volatile uint32_t* first;  // first chunk index of the CTA
    volatile uint32_t* abort;  // raised by a wait that gave up
    uint8_t* ctx;              // kCtxBytes for batch_cta
    volatile unsigned long long* limit_ns;  // the waits' time limit
};

__device__ __forceinline__ Handoff handoff_at(uint8_t* smem, uint32_t part_off, uint32_t sync_off)
{
    uint8_t* s = smem + sync_off;
    return Handoff{reinterpret_cast<uint4*>(smem + part_off), reinterpret_cast<uint64_t*>(s),
                   reinterpret_cast<uint64_t*>(s + 16), reinterpret_cast<volatile uint32_t*>(s + 32),
                   reinterpret_cast<volatile uint32_t*>(s + 40), reinterpret_cast<volatile uint32_t*>(s + 44),
                   s + 48, reinterpret_cast<volatile unsigned long long*>(s + 88)};
}

static_assert(48 + kCtxBytes <= 88 && 88 + 8 <= kHandoffSyncBytes, "hand-off shared words overlap");

// Thread 0, before the CTA's first barrier.
__device__ __forceinline__ void handoff_init(const Handoff& h, unsigned long long wait_ns)
{
    mbar_init(h.full, kHornerThreads / 32);
    mbar_init(h.full + 1, kHornerThreads / 32);
    mbar_init(h.empty, 1);
    mbar_init(h.empty + 1, 1);
    *h.abort = 0u;
    *h.limit_ns = wait_ns;
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
    if (!__all_sync(0xffffffffu, mbar_wait(h.empty + b, parity ^ 1u, h.abort, h.limit_ns))) {
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
    if (!__all_sync(0xffffffffu, mbar_wait(h.full + b, parity, h.abort, h.limit_ns))) {
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
    if (!__all_sync(0xffffffffu, mbar_wait(h.full + b, (j >> 1) & 1u, h.abort, h.limit_ns))) {
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

// Work-kernel epilogue of the chunk phase (all threads): a CTA whose hand-off
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

// Item index of the small object at queue position k: the buckets are handed
// out largest first (bucket kSmallBuckets - 1 down to 0), each from its own
// list region of `count` entries.
__device__ __forceinline__ uint32_t small_item(const BatchArgs& a, const BatchHeader* hdr, uint32_t k)
{
    const uint32_t* lists = reinterpret_cast<const uint32_t*>(a.ws + batch_small_offset(a.count));
    int b = kSmallBuckets - 1;
    for (; b > 0; --b) {
        const uint32_t n = hdr->small_bucket[b];
        if (k < n) {
            break;
        }
        k -= n;
    }
    return lists[static_cast<size_t>(b) * a.count + k];
}

// ------------------------------------------------------------------ seal

// Row warps: segments of one alignment class from the cursor on; returns
// true when the next segment has another class, false when the queue is
// exhausted (or a hand-off gave up). Per-segment values are loaded where they
// are used so that only the cursor stays live across the rows.
template <int SQ, bool PT>
__device__ __forceinline__ bool seal_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c, const Handoff& h,
                                           const WalkSlot& ws, int cls)
{
    const uint4* ft = reinterpret_cast<const uint4*>(smem + kSealBatchFold);
    for (;;) {
        uint4 q;
        {
            const Cursor cur = walk_cursor(ws);
            const Segment sg = segment_at(c, cur);
            *walk_word(ws, 1) = sg.last ? kChunkEnd : cur.k + 1;
            const BatchItem* it = a.items + sg.item;
            const uint64_t P = it->plen;
            uint8_t* frame = it->dst;
            const uint32_t ivw[3] = {it->iv[0], it->iv[1], it->iv[2]};
            if (sg.r0 == 0 && c.tid == 0) {
                frame[0] = 1;
                for (int b = 0; b < 12; ++b) {
                    frame[1 + b] = static_cast<uint8_t>(ivw[b >> 2] >> (8 * (b & 3)));
                }
            }
            int sq;
            uint32_t store_r;
            store_class(frame + 13, sq, store_r);  // sq == SQ for this class
            (void)sq;
            const SealTile t{it->src, frame + 13, P, segment_base(sg, P), static_cast<int64_t>(sg.r1 - sg.r0),
                             {ivw[0] ^ a.rk[0], ivw[1] ^ a.rk[1], ivw[2] ^ a.rk[2]}, store_r};
            q = seal_rows<SQ, PT>(t, a.rk, a.kt.gh_pow2, c.tid, c.lane);
        }
        const bool chunk_done = *walk_word(ws, 1) == kChunkEnd;
        uint32_t taken = 0;
        if (chunk_done && c.tid == 0) {
            taken = atomicAdd(&c.hdr->next_chunk[0], 1u);
        }
        const uint4 v = warp_fold_pairs<true>(q, ft, c.lane);
        const uint32_t j = *walk_word(ws, 2);
        uint32_t next;
        if (!row_handoff(h, j, v, taken, c, next)) {
            return false;
        }
        *walk_word(ws, 2) = j + 1;
        if (chunk_done && !walk_open(c, next, ws)) {
            return false;
        }
        if (cursor_class(c, walk_cursor(ws)) != cls) {
            return true;
        }
    }
}

// CTR pass of a two-pass seal (seal_batch_kernel's row warps only): each
// segment's rows are encrypted into its frame (seal_rows without the GHASH
// chain), the segment at row 0 also writes the header. Chunks come from
// queue 0; the row warps share the next chunk index through shared memory
// (the unused hand-off buffers) behind named barrier 1, which the power warp
// does not take part in.
template <int SQ, bool PT>
__device__ __forceinline__ bool seal_ctr_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c, Cursor& cur,
                                               int cls, uint32_t& round)
{
    volatile uint32_t* next_s = reinterpret_cast<volatile uint32_t*>(smem + kSealBatchHandoff);
    for (;;) {
        const Segment sg = segment_at(c, cur);
        {
            const BatchItem* it = a.items + sg.item;
            const uint64_t P = it->plen;
            uint8_t* frame = it->dst;
            const uint32_t ivw[3] = {it->iv[0], it->iv[1], it->iv[2]};
            if (sg.r0 == 0 && c.tid == 0) {
                frame[0] = 1;
                for (int b = 0; b < 12; ++b) {
                    frame[1 + b] = static_cast<uint8_t>(ivw[b >> 2] >> (8 * (b & 3)));
                }
            }
            int sq;
            uint32_t store_r;
            store_class(frame + 13, sq, store_r);  // sq == SQ for this class
            (void)sq;
            const SealTile t{it->src, frame + 13, P, segment_base(sg, P), static_cast<int64_t>(sg.r1 - sg.r0),
                             {ivw[0] ^ a.rk[0], ivw[1] ^ a.rk[1], ivw[2] ^ a.rk[2]}, store_r};
            seal_rows<SQ, PT, false>(t, a.rk, a.kt.gh_pow2, c.tid, c.lane);
        }
        if (cursor_step(cur, sg)) {
            if (c.tid == 0) {
                next_s[round & 1] = atomicAdd(&c.hdr->next_chunk[0], 1u);
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kHornerThreads) : "memory");
            const uint32_t next = next_s[round & 1];
            ++round;
            if (!cursor_open(c, next, cur)) {
                return false;
            }
        }
        if (cursor_class(c, cur) != cls) {
            return true;
        }
    }
}

__device__ __forceinline__ void seal_ctr_walk(uint8_t* smem, const BatchArgs& a, const BatchCta& c, uint32_t chunk)
{
    Cursor cur;
    bool more = cursor_open(c, chunk, cur);
    uint32_t round = 0;  // parity of the shared next-chunk entry
    while (more) {
        const int cls = cursor_class(c, cur);
        switch (cls) {
        case 0: more = seal_ctr_class<0, false>(smem, a, c, cur, cls, round); break;
        case 1: more = seal_ctr_class<0, true>(smem, a, c, cur, cls, round); break;
        case 2: more = seal_ctr_class<1, false>(smem, a, c, cur, cls, round); break;
        case 3: more = seal_ctr_class<1, true>(smem, a, c, cur, cls, round); break;
        case 4: more = seal_ctr_class<2, false>(smem, a, c, cur, cls, round); break;
        case 5: more = seal_ctr_class<2, true>(smem, a, c, cur, cls, round); break;
        case 6: more = seal_ctr_class<3, false>(smem, a, c, cur, cls, round); break;
        case 7: more = seal_ctr_class<3, true>(smem, a, c, cur, cls, round); break;
        case 8: more = seal_ctr_class<4, false>(smem, a, c, cur, cls, round); break;
        default: more = seal_ctr_class<4, true>(smem, a, c, cur, cls, round); break;
        }
    }
}

// Power warp of the batched seal, over the same segments as the row warps:
// E_K(J0), L*H and the basis of H^d while the segment's rows run, then the
// fold levels 4..8 (the key's global tables), the object's sum and, once the
// object's last segment is in, its tag.
__device__ __forceinline__ void seal_power_loop(const BatchArgs& a, const BatchCta& c, const Handoff& h,
                                                uint32_t chunk)
{
    Cursor cur;
    bool more = cursor_open(c, chunk, cur) && a.stall == 0u;
    for (uint32_t j = 0; more; ++j) {
        const Segment sg = segment_at(c, cur);
        Slot* slot = cta_slots(c) + sg.item;
        const BatchItem* it = a.items + sg.item;
        const uint32_t G = slot->aux[1];
        const uint64_t P = it->plen;
        const uint32_t ivw[3] = {it->iv[0], it->iv[1], it->iv[2]};
        uint4 ej0, lh;
        unsigned long long uhi, ulo;
        seal_power(ivw, a.rk, P, segment_power(sg), a.kt.gh_pow2, c.lane, ej0, lh, uhi, ulo);
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
        if (cursor_step(cur, sg)) {
            more = cursor_open(c, next, cur);
        }
    }
}

__global__ void __launch_bounds__(kSealThreads, 1) seal_batch_kernel(const BatchArgs a)
{
    uint8_t* const smem = layout_smem();
    const int tid = threadIdx.x;
    pdl_release();
    fill_aes_smem(smem + kSealAes, a.kt.aes_t);
    fill_gh_smem(smem + kSealGh, a.kt.gh_pow2 + kSealChainLog2 * 512);
    fill_small_fold(smem, a.kt.gh_pow2);
    const Handoff h = handoff_at(smem, kSealBatchHandoff, kSealBatchSync);
    if (tid == 0) {
        handoff_init(h, a.wait_ns);
    }
    pdl_wait();  // the plan kernel's workspace
    const BatchCta c = batch_cta(a, h.ctx, tid);
    const uint32_t chunk = first_chunk(h.first, c, 0);
    if (c.hdr->seal_two_pass != 0u) {
        // CTR pass of a two-pass seal: the row warps encrypt the chunks
        // (seal_ghash_batch_kernel hashes them next); the power warp waits
        // for the small objects
        if (c.warp != kPowerWarp) {
            seal_ctr_walk(smem, a, c, chunk);
        }
    } else if (c.warp == kPowerWarp) {
        seal_power_loop(a, c, h, chunk);
    } else {
        const WalkSlot ws{smem + kSealBatchWalk};
        *walk_word(ws, 2) = 0;
        bool more = walk_open(c, chunk, ws);
        while (more) {
            const int cls = cursor_class(c, walk_cursor(ws));
            switch (cls) {
            case 0: more = seal_class<0, false>(smem, a, c, h, ws, cls); break;
            case 1: more = seal_class<0, true>(smem, a, c, h, ws, cls); break;
            case 2: more = seal_class<1, false>(smem, a, c, h, ws, cls); break;
            case 3: more = seal_class<1, true>(smem, a, c, h, ws, cls); break;
            case 4: more = seal_class<2, false>(smem, a, c, h, ws, cls); break;
            case 5: more = seal_class<2, true>(smem, a, c, h, ws, cls); break;
            case 6: more = seal_class<3, false>(smem, a, c, h, ws, cls); break;
            case 7: more = seal_class<3, true>(smem, a, c, h, ws, cls); break;
            case 8: more = seal_class<4, false>(smem, a, c, h, ws, cls); break;
            default: more = seal_class<4, true>(smem, a, c, h, ws, cls); break;
            }
        }
    }
    if (handoff_failed(h, c)) {
        return;
    }

    // Small objects, one warp each, once the chunks are gone: H^32 over the
    // chain table (the fold slots already hold H^8, H^1, H^2, H^4).
    const uint32_t small_count = c.hdr->small_count;
    if (small_count == 0) {
        return;
    }
    fill_gh_smem(smem + kSmallGh, a.kt.gh_pow2 + 5 * 512);
    __syncthreads();
    for (;;) {
        uint32_t k = 0;
        if (c.lane == 0) {
            k = atomicAdd(&c.hdr->small_next[0], 1u);
        }
        k = __shfl_sync(0xffffffffu, k, 0);
        if (k >= small_count) {
            break;
        }
        seal_object_warp(a.items + small_item(a, c.hdr, k), a.rk, a.kt.gh_pow2, smem, c.lane);
    }
}

// ------------------------------------------------------------------ open

// GHASH pass of the batched open (SEAL = false: frames are the descriptors'
// sources, the power warp checks tags) and of the batched seal (SEAL = true:
// frames are the destinations, written by seal_ctr_batch_kernel earlier on
// the stream, and the power warp writes their tags). The ciphertext load
// class LQ of a segment: open takes it from the plan's alignment class; a
// seal object's class codes its store funnel, so the seal pass derives LQ
// from the frame address.
template <bool SEAL>
__device__ __forceinline__ const uint8_t* ghash_frame(const BatchItem* it)
{
    return SEAL ? it->dst : it->src;
}

template <bool SEAL>
__device__ __forceinline__ int ghash_load_class(const BatchArgs& a, const BatchCta& c, const Cursor& cur)
{
    if constexpr (SEAL) {
        int lq;
        uint32_t r;
        load_class(ghash_frame<true>(a.items + cta_objs(c)[cur.k].item) + 13, lq, r);
        return lq;
    } else {
        return cursor_class(c, cur) >> 1;
    }
}

// Row warps of the GHASH pass: segments whose frames share load class LQ;
// same contract as seal_class.
template <bool SEAL, int LQ>
__device__ __forceinline__ bool ghash_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c, const Handoff& h,
                                            const WalkSlot& ws, int pass)
{
    const uint4* ft = reinterpret_cast<const uint4*>(smem + kGhPassFold);
    for (;;) {
        uint4 q;
        {
            const Cursor cur = walk_cursor(ws);
            const Segment sg = segment_at(c, cur);
            *walk_word(ws, 1) = sg.last ? kChunkEnd : cur.k + 1;
            const BatchItem* it = a.items + sg.item;
            const uint64_t P = it->plen;
            const uint8_t* frame = ghash_frame<SEAL>(it);
            int lq;
            uint32_t load_r;
            load_class(frame + 13, lq, load_r);  // lq == LQ for this class
            (void)lq;
            const OpenTile t{frame, it->capacity, P, segment_base(sg, P), static_cast<int64_t>(sg.r1 - sg.r0),
                             load_r};
            q = open_ghash_rows<LQ, kOpenBatchChains, kOpenBatchAluChains, kOpenBatchStepRows, kGhashTable5, kGhPassGh>(
                t, reinterpret_cast<const uint4*>(smem + kGhPassHt), &a.open_cm, c.tid, c.lane);
        }
        const bool chunk_done = *walk_word(ws, 1) == kChunkEnd;
        uint32_t taken = 0;
        if (chunk_done && c.tid == 0) {
            taken = atomicAdd(&c.hdr->next_chunk[pass], 1u);
        }
        const uint4 v = warp_fold_pairs<false>(q, ft, c.lane);
        const uint32_t j = *walk_word(ws, 2);
        uint32_t next;
        if (!row_handoff(h, j, v, taken, c, next)) {
            return false;
        }
        *walk_word(ws, 2) = j + 1;
        if (chunk_done && !walk_open(c, next, ws)) {
            return false;
        }
        if (ghash_load_class<SEAL>(a, c, walk_cursor(ws)) != LQ) {
            return true;
        }
    }
}

// Power warp of the GHASH pass: E_K(J0) (IV from the frame), L*H and the
// basis of H^d while the rows run, then fold levels 4..8 (shared tables), the
// object's sum and, once its last segment is in, the tag (seal) or the
// verdict (open: auth_ok and the object's slot).
template <bool SEAL>
__device__ __forceinline__ void ghash_power_loop(const uint8_t* smem, const BatchArgs& a, const BatchCta& c,
                                                 const Handoff& h, uint32_t chunk)
{
    const uint4* t4 = (kGhPassFoldLevels == kFoldLevels ? reinterpret_cast<const uint4*>(smem + kGhPassFold)
                                                         : a.kt.gh_pow2) +
                      4 * 512;
    Cursor cur;
    bool more = cursor_open(c, chunk, cur) && (!SEAL || a.stall == 0u);
    for (uint32_t j = 0; more; ++j) {
        const Segment sg = segment_at(c, cur);
        Slot* slot = cta_slots(c) + sg.item;
        const BatchItem* it = a.items + sg.item;
        const uint32_t G = slot->aux[1];
        const uint64_t P = it->plen;
        const uint8_t* frame = ghash_frame<SEAL>(it);
        uint4 ej0, lh;
        unsigned long long uhi, ulo;
        open_power(frame, a.kt.aes_t, a.rk, P, segment_power(sg), a.kt.gh_pow2, c.lane, ej0, lh, uhi, ulo);
        uint4 v;
        uint32_t next;
        if (!power_take(h, j, c.lane, v, next)) {
            return;
        }
        const uint4 fold = power_fold(v, t4, c.lane);
        unsigned long long shi, slo;
        if (batch_object_sum(slot, G, fold, uhi, ulo, c.lane, shi, slo)) {
            if constexpr (SEAL) {
                const uint4 tag = xor4(xor4(be_to_raw(shi, slo), lh), ej0);
                if (c.lane < 16) {
                    it->dst[13 + P + c.lane] = static_cast<uint8_t>(byte_of(tag, c.lane));
                }
            } else if (c.lane == 0) {
                const int ok = open_verdict(frame, P, shi, slo, lh, ej0);
                *it->auth_ok = ok;
                slot->aux[2] = static_cast<unsigned int>(ok);
            }
        }
        if (cursor_step(cur, sg)) {
            more = cursor_open(c, next, cur);
        }
    }
}

// The GHASH pass's CTA: the single-object open layout (the chain table,
// fold tables H^1..H^512, compact H^512) plus the hand-off; `pass` = the
// chunk queue this pass takes (open: the first pass, seal: the second).
template <bool SEAL>
__device__ __forceinline__ void ghash_batch_cta(const BatchArgs& a, int pass)
{
    uint8_t* const smem = layout_smem();
    const int tid = threadIdx.x;
    pdl_release();
    if constexpr (SEAL) {
        // the plan may have chosen the fused seal, whose kernel wrote the
        // tags already: read its choice before any table fill, so that a
        // pass with nothing to do ends at once
        pdl_wait();
        if (reinterpret_cast<const volatile BatchHeader*>(a.ws)->seal_two_pass == 0u) {
            return;
        }
    }
    if constexpr (kGhashTable5) {
        fill_gh5_smem(smem + kGhPassGh, a.kt.gh_chain5);
    } else {
        fill_gh_smem(smem + kGhPassGh, a.kt.gh_chain);
    }
    fill_smem<kGhPassFoldLevels * 512>(reinterpret_cast<uint4*>(smem + kGhPassFold), a.kt.gh_pow2);
    fill_smem<512>(reinterpret_cast<uint4*>(smem + kGhPassHt), a.kt.gh_pow2 + kFoldLevels * 512);
    const Handoff h = handoff_at(smem, kOpenBatchHandoff, kOpenBatchSync);
    if (tid == 0) {
        handoff_init(h, a.wait_ns);
    }
    if constexpr (!SEAL) {
        pdl_wait();  // the plan's workspace
    }
    const BatchCta c = batch_cta(a, h.ctx, tid);
    const uint32_t chunk = first_chunk(h.first, c, pass);
    if (c.warp == kPowerWarp) {
        ghash_power_loop<SEAL>(smem, a, c, h, chunk);
    } else {
        const WalkSlot ws{smem + kOpenBatchWalk};
        *walk_word(ws, 2) = 0;
        bool more = walk_open(c, chunk, ws);
        while (more) {
            switch (ghash_load_class<SEAL>(a, c, walk_cursor(ws))) {  // the GHASH pass reads only the frames
            case 0: more = ghash_class<SEAL, 0>(smem, a, c, h, ws, pass); break;
            case 1: more = ghash_class<SEAL, 1>(smem, a, c, h, ws, pass); break;
            case 2: more = ghash_class<SEAL, 2>(smem, a, c, h, ws, pass); break;
            case 3: more = ghash_class<SEAL, 3>(smem, a, c, h, ws, pass); break;
            default: more = ghash_class<SEAL, 4>(smem, a, c, h, ws, pass); break;
            }
        }
    }
    handoff_failed(h, c);
}

__global__ void __launch_bounds__(kSealThreads, 1) open_ghash_batch_kernel(const BatchArgs a)
{
    ghash_batch_cta<false>(a, 0);
}

__global__ void __launch_bounds__(kSealThreads, 1) seal_ghash_batch_kernel(const BatchArgs a)
{
    ghash_batch_cta<true>(a, 1);
}

// Gated CTR over the same row space (rows of kCtrThreads = kHornerThreads
// blocks), chunks from a second queue. Each segment reads its object's
// verdict, written by open_ghash_batch_kernel earlier on the stream:
// authentic -> decrypt, otherwise zero the segment's plaintext bytes. Thread
// 0 takes the next chunk after the rows of a chunk's last segment; it goes
// through a two-entry shared buffer so one barrier per chunk suffices.
template <int LQ, bool PT>
__device__ __forceinline__ bool ctr_class(uint8_t* smem, const BatchArgs& a, const BatchCta& c, Cursor& cur,
                                          int cls, uint32_t& round)
{
    static_assert(kCtrThreads == kHornerThreads, "CTR segments reuse the GHASH rows");
    volatile uint32_t* next_s = reinterpret_cast<volatile uint32_t*>(smem + kCtrBatchMisc);
    for (;;) {
        const Segment sg = segment_at(c, cur);
        {
            const BatchItem* it = a.items + sg.item;
            const int ok = static_cast<int>(cta_slots(c)[sg.item].aux[2]);
            const uint64_t P = it->plen;
            const uint8_t* frame = it->src;
            int lq;
            uint32_t load_r;
            load_class(frame + 13, lq, load_r);  // lq == LQ for this class
            (void)lq;
            CtrTile t{frame, it->capacity, it->dst, P, segment_base(sg, P), static_cast<int64_t>(sg.r1 - sg.r0),
                      {0u, 0u, 0u}, load_r};
            if (!ok) {
                ctr_zero_rows<PT>(t, c.tid);
            } else {
                const uint4 iv = load_bytes(frame + 1, 12);
                t.s012[0] = iv.x ^ a.rk[0];
                t.s012[1] = iv.y ^ a.rk[1];
                t.s012[2] = iv.z ^ a.rk[2];
                ctr_rows<LQ, PT>(t, a.rk, c.tid, c.lane);
            }
        }
        if (cursor_step(cur, sg)) {
            if (c.tid == 0) {
                next_s[round & 1] = atomicAdd(&c.hdr->next_chunk[1], 1u);
            }
            __syncthreads();
            const uint32_t next = next_s[round & 1];
            ++round;
            if (!cursor_open(c, next, cur)) {
                return false;
            }
        }
        if (cursor_class(c, cur) != cls) {
            return true;
        }
    }
}

__global__ void __launch_bounds__(kCtrThreads, 1) open_ctr_batch_kernel(const BatchArgs a)
{
    uint8_t* const smem = layout_smem();
    const int tid = threadIdx.x;
    pdl_release();
    fill_aes_smem(smem, a.kt.aes_t);
    small_fill_open_tables(smem, a.kt.gh_pow2);
    pdl_wait();  // the verdicts of the GHASH pass
    const BatchCta c = batch_cta(a, smem + kCtrBatchMisc + 16, tid);
    const uint32_t chunk = first_chunk(reinterpret_cast<volatile uint32_t*>(smem + kCtrBatchMisc) + 2, c, 1);
    Cursor cur;
    bool more = cursor_open(c, chunk, cur);
    uint32_t round = 0;  // parity of the shared buffer entry, continued across classes
    while (more) {
        const int cls = cursor_class(c, cur);
        switch (cls) {
        case 0: more = ctr_class<0, false>(smem, a, c, cur, cls, round); break;
        case 1: more = ctr_class<0, true>(smem, a, c, cur, cls, round); break;
        case 2: more = ctr_class<1, false>(smem, a, c, cur, cls, round); break;
        case 3: more = ctr_class<1, true>(smem, a, c, cur, cls, round); break;
        case 4: more = ctr_class<2, false>(smem, a, c, cur, cls, round); break;
        case 5: more = ctr_class<2, true>(smem, a, c, cur, cls, round); break;
        case 6: more = ctr_class<3, false>(smem, a, c, cur, cls, round); break;
        case 7: more = ctr_class<3, true>(smem, a, c, cur, cls, round); break;
        case 8: more = ctr_class<4, false>(smem, a, c, cur, cls, round); break;
        default: more = ctr_class<4, true>(smem, a, c, cur, cls, round); break;
        }
    }

    // Small objects: one warp opens a whole object (GHASH, tag check, CTR),
    // so its plaintext waits for nothing outside the warp.
    const uint32_t small_count = c.hdr->small_count;
    for (;;) {
        uint32_t k = 0;
        if (c.lane == 0) {
            k = atomicAdd(&c.hdr->small_next[1], 1u);
        }
        k = __shfl_sync(0xffffffffu, k, 0);
        if (k >= small_count) {
            break;
        }
        open_object_warp(a.items + small_item(a, c.hdr, k), a.rk, a.kt.gh_pow2, smem, c.lane);
    }
}

}  // namespace dev
}  // namespace confkv
