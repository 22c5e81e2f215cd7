// Device code for the B200 AES-128-GCM engine: AES rounds on replicated
// T-tables in shared memory, 4-bit GHASH tables, warp-parallel GF(2^128)
// helpers, and the seal / open-GHASH / open-CTR kernels.
//
// Register layout used throughout: a 16-byte block is four little-endian
// 32-bit words (word c = bytes 4c..4c+3, byte 4c in the low bits). AES state
// word c is state column c (row r = byte r). GHASH values are kept as raw
// block bytes in the same layout; the tables encode the SP 800-38D bit order.
#pragma once

#include <cstdint>
#include <utility>

#include "clmul.cuh"
#include "gh5.cuh"

namespace confkv {
namespace dev {

constexpr int kHornerThreads = 512;                 // threads running GHASH rows per CTA
constexpr int kHornerLog2 = 9;                      // log2(kHornerThreads)
constexpr int kFoldLevels = kHornerLog2;
constexpr int kSealChains = 1;                      // GHASH chains per thread in seal
constexpr int kSealChainLog2 = kHornerLog2;         // chain multiplier H^kHornerThreads
constexpr int kOpenChainLog2 = kHornerLog2 + 1;     // per-object open, objects below kOpenWindowMinBytes: H^(2 T)
// The batched GHASH passes (open, and the two-pass seal) run
// kOpenBatchChains chains per thread (multiplier H^(kOpenBatchChains T), a
// compact table of its own in the key tables); the last
// kOpenBatchAluChains of them multiply on the integer pipes (clmul.cuh)
// instead of the shared-memory tables, so the two share the GHASH work. A
// table multiply costs 4 shared-memory wavefronts per block with 4-bit
// tables, 2.75 with the 6-bit windows the batched passes use, and ~110 ALU
// instructions; an integer-pipe multiply ~310 ALU and ~150 FMA-pipe
// instructions (ncu, B200). Measured on 32 x 32 MiB (open GB/s) with 4-bit
// tables: tables only 502; one chain in four 549; one in three 538 and two
// in five 511 (both lose although the shared-memory pipe still binds at one
// in four: with fewer table rows between its steps the integer-pipe chain's
// latency shows); one in two 495. With 6-bit windows: one in four 585,
// tables only 565, one in five 572, one in three 540, two in five 528.
// The per-object open uses the same split for large objects and two 4-bit
// table chains below kOpenWindowMinBytes (OpenLayout).
constexpr int kOpenBatchChains = 4;
constexpr int kOpenBatchAluChains = 1;
constexpr int kOpenBatchStepRows = 1;               // interior rows read (and prefetched) at a time
constexpr int kPowerWarp = kHornerThreads / 32;     // warp index of the power warp
constexpr int kSealThreads = kHornerThreads + 32;
constexpr int kCtrThreads = 512;

// Shared-window address at which every kernel's shared-memory layout begins.
// Dynamic shared memory starts after the block's reserved bytes (1 KiB on
// sm_100a with this driver); a kernel skips from there to kSmemLayoutBase
// (layout_smem), and the host adds that gap to every launch (layout_pad in
// host_common.h). Hot-loop table loads put kSmemLayoutBase in the LDS
// immediate field, so the PRMT-formed offset needs no add, whatever the
// reserve is, up to kSmemLayoutBase. Adding a base register to each lookup
// instead would put 133 more ALU instructions on every AES-CTR block.
constexpr uint32_t kSmemLayoutBase = 0x800;
constexpr uint32_t kSmemOptInLimit = 227u * 1024u;
// Room for the gap of today's 1 KiB reserve in every kernel's budget.
constexpr uint32_t kSmemGapToday = kSmemLayoutBase - 0x400u;

// Shared-memory regions (byte offsets from the start of the layout).
// AES T-tables: two 64 KiB regions; row x (256 B) of region 0 holds T0[x] for
// lanes 0..31 then T1[x] for lanes 0..31; region 1 holds T2 and T3. A lookup
// address is formed by one PRMT: byte 0 = table half + lane, byte 1 = index.
constexpr uint32_t kAesBytes = 128u << 10;
// GHASH main table: row (j << 4 | v) (256 B) holds, for byte j of the block and
// nibble value v, 8 replicas (16 B each) of the low-nibble entry then 8 of the
// high-nibble entry. Lane l reads replica l & 7, so the 8 lanes of one LDS.128
// phase hit 8 distinct bank groups.
constexpr uint32_t kGhBytes = 64u << 10;
constexpr uint32_t kPartBytes = kHornerThreads * 16;
// After the main loop the fold tables H^(2^l), l < kFoldLevels (8 KiB each),
// are staged over a table region that is no longer read.
constexpr uint32_t kFoldBytes = kFoldLevels * 8192u;

constexpr int kSealFoldSmemLevels = 3;             // fold levels whose tables seal keeps in smem
constexpr uint32_t kSealAes = 0;
constexpr uint32_t kSealGh = kSealAes + kAesBytes;
constexpr uint32_t kSealPart = kSealGh + kGhBytes;
constexpr uint32_t kSealFold = kSealPart + kPartBytes;
constexpr uint32_t kSealMisc = kSealFold + kSealFoldSmemLevels * 8192u;
constexpr uint32_t kSealSmem = kSealMisc + 64;

// Per-object open GHASH, two designs (OpenLayout<WIN>), chosen per call by
// the object's size:
//   WIN = false (objects under kOpenWindowMinBytes): two chains on the
//     replicated 4-bit table of H^(2 T); every fold table in shared memory.
//   WIN = true: the batched GHASH passes' split, kOpenBatchChains chains
//     (multiplier H^(4 T)), the first on its replicated 6-bit window table
//     (gh5.cuh), the last kOpenBatchAluChains on the integer pipes; the fold
//     tables of levels 0..3 in shared memory, levels 4..8 from the key's
//     global tables (the window table leaves no room for them).
// The window table costs every CTA a 176 KiB fill, which small objects do
// not earn back. Measured on B200, per-object open GB/s, 4-bit -> window:
// 32 MiB 402 -> 388, 48 MiB 432 -> 431, 64 MiB 449 -> 465, 128 MiB 478 ->
// 522, 256 MiB 496 -> 556, 1 GiB 510 -> 588.
template <bool WIN>
struct OpenLayout {
    static constexpr int kChains = WIN ? kOpenBatchChains : 2;
    static constexpr int kAluChains = WIN ? kOpenBatchAluChains : 0;
    static constexpr int kStepRows = WIN ? kOpenBatchStepRows : 2;
    static constexpr int kFoldSmemLevels = WIN ? 4 : kFoldLevels;
    static constexpr uint32_t kGh = 0;
    static constexpr uint32_t kFold = kGh + (WIN ? static_cast<uint32_t>(kGh5RepBytes) : kGhBytes);
    static constexpr uint32_t kHt = kFold + static_cast<uint32_t>(kFoldSmemLevels) * 8192u;  // H^kHornerThreads
    static constexpr uint32_t kPart = kHt + 8192u;
    // the compact AES T-tables for the power warp's E_K(J0) (4-bit layout only)
    static constexpr uint32_t kAesC = kPart + kPartBytes + 64;
    static constexpr uint32_t kSmem = kAesC + (WIN ? 0u : 4096u);
    static_assert(kSmem + kSmemGapToday <= kSmemOptInLimit, "per-object open shared memory exceeds the per-block limit");
};
constexpr uint64_t kOpenWindowMinBytes = 48ull << 20;
// Per-object seal of objects from kSealTwoPassMinBytes on: a CTR-only pass
// (seal_ctr_kernel, 512 threads), then the window-table GHASH kernel of the
// per-object open over the frame's ciphertext, which writes the tag. The
// second pass re-reads the ciphertext and adds a launch, which pays from
// about 80 MiB. Measured on B200, per-object seal GB/s, fused -> two passes:
// 48 MiB 441 -> 417, 64 MiB 452 -> 448, 96 MiB 466 -> 481, 128 MiB 476 ->
// 495, 256 MiB 487 -> 537, 512 MiB 493 -> 556, 1 GiB 496 -> 569.
constexpr uint64_t kSealTwoPassMinBytes = 80ull << 20;
constexpr uint32_t kOpenGh = 0;  // shared offset of the chain table (both layouts)

constexpr uint32_t kCtrSmem = kAesBytes;
static_assert(kSealSmem + kSmemGapToday <= kSmemOptInLimit, "seal shared memory exceeds the per-block limit");

// Per-call accumulation slot (32 bytes). The last CTA of a call resets
// acc_hi, acc_lo and ticket. Batched calls keep one slot per object and its
// tile plan in aux: {J, G, authentication verdict}.
struct Slot {
    unsigned long long acc_hi;
    unsigned long long acc_lo;
    unsigned int ticket;
    unsigned int aux[3];
};

struct KeyTables {
    const uint32_t* aes_t;   // T0..T3, 4 x 256 words
    const uint4* gh_pow2;    // compact 4-bit tables (512 entries) for H^(2^k), k = 0..35
    const uint4* gh_chain;   // compact 4-bit table of the batched GHASH passes' chain multiplier H^(kOpenBatchChains T)
    const uint4* gh_chain5;  // the same multiplier's window table (kGhW bits, gh5.cuh)
};

struct SealArgs {
    const uint8_t* src;
    uint8_t* frame;
    uint64_t plen;
    uint32_t nblocks;
    uint32_t iters;     // Horner iterations per CTA (J)
    uint32_t grid;      // CTAs (G)
    uint32_t store_r;   // byte part of the ciphertext store funnel
    uint32_t ivw[3];    // IV as little-endian words
    uint32_t rk[44];
    KeyTables kt;
    Slot* slot;
};

struct OpenArgs {
    const uint8_t* frame;
    uint64_t frame_len;
    uint64_t plen;
    uint32_t nblocks;
    uint32_t iters;
    uint32_t grid;
    uint32_t load_r;    // byte part of the ciphertext load funnel
    uint32_t rk[44];
    KeyTables kt;
    Slot* slot;
    int* auth_ok;
    ClmulConst cm;      // the chain multiplier for the integer-pipe chain (OpenLayout<true>)
    uint8_t* tag_out;   // two-pass seal: the frame whose tag the GHASH kernel writes (open: null)
};

struct CtrArgs {
    const uint8_t* frame;
    uint64_t frame_len;
    uint8_t* dst;
    uint64_t plen;
    uint32_t nblocks;
    uint32_t load_r;
    uint32_t rows_per_cta;  // rows of kCtrThreads blocks per CTA
    uint32_t rk[44];
    const uint32_t* aes_t;
    const int* auth_ok;
};

// ------------------------------------------------ programmatic dependent launch
//
// The single-object kernels are launched with programmatic stream
// serialization: pdl_release() at the top of every CTA lets the next kernel
// on the stream launch once all of this grid's CTAs run, so its CTAs take
// SMs as this grid's CTAs exit and fill their shared tables (key tables
// only, written once by key_create) while this grid drains. Every access to
// memory another kernel of the stream may read or write -- objects, frames,
// slots, auth_ok -- comes after pdl_wait(), which returns once the previous
// grid has completed and its writes are visible (at once when there is no
// programmatic predecessor).
__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_release()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------ shared-memory mbarriers
//
// Warps of one CTA hand data to one another through shared memory guarded by
// mbarriers (arrive = release, completed wait = acquire, CTA scope). Every
// wait is bounded: it gives up after kWaitLimitNs of %globaltimer (or
// kWaitLimitPolls polls) or as soon as another thread of the CTA has given up,
// raising the CTA's shared abort word, so a broken hand-off ends the kernel
// with an error instead of hanging it. The limit is far above any legitimate
// wait (a wait lasts at most one tile of rows, milliseconds).
constexpr unsigned long long kWaitLimitNs = 10ull * 1000ull * 1000ull * 1000ull;
constexpr uint32_t kWaitLimitPolls = 1u << 30;

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The start of the kernel's shared layout: window address kSmemLayoutBase,
// inside the block's dynamic shared memory because the host sized the launch
// to include the gap (layout_pad). A constant shared address, so every
// region's address folds into its instructions' immediates.
__device__ __forceinline__ uint8_t* layout_smem()
{
    return static_cast<uint8_t*>(__cvta_shared_to_generic(kSmemLayoutBase));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

// True once the phase of `bar` with parity `parity` has completed.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase of `bar` with parity `parity`; false when the
// limit ran out (the caller's thread raises *abort) or *abort was raised.
// *limit_ns is the time limit (kWaitLimitNs unless a test shortens it); it is
// read only once the first test has failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                          const volatile unsigned long long* limit_ns)
{
    if (mbar_test(bar, parity)) {
        return true;
    }
    const unsigned long long limit = *limit_ns;
    const unsigned long long t0 = global_ns();
    for (uint32_t polls = 0; polls < kWaitLimitPolls; ++polls) {
        if (mbar_test(bar, parity)) {
            return true;
        }
        if (*abort != 0u) {
            return false;
        }
        if (global_ns() - t0 > limit) {
            break;
        }
    }
    *abort = 1u;
    return false;
}

// Device view of lmcache_gpu_aesgcm_batch_item (include/gpu_aesgcm_api.h).
struct BatchItem {
    const uint8_t* src;   // seal: plaintext; open: frame
    uint8_t* dst;         // seal: frame; open: plaintext
    uint64_t plen;
    uint64_t capacity;    // seal: dst capacity; open: frame length
    int* auth_ok;         // open only
    uint32_t iv[3];       // seal only: IV bytes as little-endian words
    int32_t status;       // written by the plan: 0 or ERR_ARGUMENT
    uint64_t reserved;
};
static_assert(sizeof(BatchItem) == 64, "batch descriptor is 64 bytes");

// ---------------------------------------------------------------- helpers

__device__ __forceinline__ uint32_t bswap32(uint32_t x)
{
    return __byte_perm(x, 0, 0x0123);
}

// Bytes r..r+3 of the little-endian pair (lo, hi); sel = r | (r+1)<<4 | ...
__device__ __forceinline__ uint32_t funnel(uint32_t lo, uint32_t hi, uint32_t sel)
{
    return __byte_perm(lo, hi, sel);
}

__host__ __device__ constexpr uint32_t funnel_sel(uint32_t r)
{
    return r | ((r + 1) << 4) | ((r + 2) << 8) | ((r + 3) << 12);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int k)
{
    return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int b)
{
    const uint32_t w = b < 4 ? v.x : b < 8 ? v.y : b < 12 ? v.z : v.w;
    return (w >> (8 * (b & 3))) & 0xffu;
}

__device__ __forceinline__ uint4 xor4(uint4 a, uint4 b)
{
    return make_uint4(a.x ^ b.x, a.y ^ b.y, a.z ^ b.z, a.w ^ b.w);
}

__device__ __forceinline__ uint4 shfl_down4(uint4 v, int d)
{
    return make_uint4(__shfl_down_sync(0xffffffffu, v.x, d), __shfl_down_sync(0xffffffffu, v.y, d),
                      __shfl_down_sync(0xffffffffu, v.z, d), __shfl_down_sync(0xffffffffu, v.w, d));
}

__device__ __forceinline__ uint4 shfl4(uint4 v, int src)
{
    return make_uint4(__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src),
                      __shfl_sync(0xffffffffu, v.z, src), __shfl_sync(0xffffffffu, v.w, src));
}

// Raw block bytes (LE words) <-> (hi, lo) big-endian halves.
__device__ __forceinline__ void raw_to_be(uint4 v, unsigned long long& hi, unsigned long long& lo)
{
    hi = (static_cast<unsigned long long>(bswap32(v.x)) << 32) | bswap32(v.y);
    lo = (static_cast<unsigned long long>(bswap32(v.z)) << 32) | bswap32(v.w);
}

__device__ __forceinline__ uint4 be_to_raw(unsigned long long hi, unsigned long long lo)
{
    return make_uint4(bswap32(static_cast<uint32_t>(hi >> 32)), bswap32(static_cast<uint32_t>(hi)),
                      bswap32(static_cast<uint32_t>(lo >> 32)), bswap32(static_cast<uint32_t>(lo)));
}

// v * x in the SP 800-38D convention (right shift, reduce by 0xE1 || 0^120).
__device__ __forceinline__ void gf_mul_x(unsigned long long& hi, unsigned long long& lo)
{
    const unsigned long long lsb = lo & 1ull;
    lo = (lo >> 1) | (hi << 63);
    hi = (hi >> 1) ^ (0xe100000000000000ull & (0ull - lsb));
}

// ------------------------------------------------------------------ AES

// Shared loads at (dynamic-shared offset `off` + region offset BASE): the
// constant part of the address rides in the instruction's immediate field.
template <uint32_t BASE>
__device__ __forceinline__ uint32_t lds32(uint32_t off)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(off), "n"(kSmemLayoutBase + BASE));
    return v;
}

template <uint32_t BASE>
__device__ __forceinline__ uint4 lds128(uint32_t off)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4+%5];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(off), "n"(kSmemLayoutBase + BASE));
    return v;
}

// One T-table lookup in the replicated shared-memory tables (region at
// dynamic offset TAB): index byte m of w, table half/lane from lb (bytes 0
// and 2 of lb pass through the PRMT).
template <uint32_t TAB>
__device__ __forceinline__ uint32_t tlook(uint32_t w, uint32_t lb, int m)
{
    return lds32<TAB>(__byte_perm(w, lb, 0x7604u | (static_cast<uint32_t>(m) << 4)));
}

// Rounds R0..10 of AES-128 on state w (the output of round R0-1) with the
// shared tables at dynamic offset TAB.
template <uint32_t TAB, int R0>
__device__ __forceinline__ void aes_rounds_from(uint32_t w[4], const uint32_t* rk, const uint32_t lb[4])
{
#pragma unroll
    for (int r = R0; r < 10; ++r) {
        uint32_t n[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            n[c] = tlook<TAB>(w[c], lb[0], 0) ^ tlook<TAB>(w[(c + 1) & 3], lb[1], 1) ^
                   tlook<TAB>(w[(c + 2) & 3], lb[2], 2) ^ tlook<TAB>(w[(c + 3) & 3], lb[3], 3) ^
                   rk[4 * r + c];
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            w[c] = n[c];
        }
    }
    uint32_t n[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        // S-box bytes taken from the table whose entry holds S[x] at the
        // byte position of the output row: T2 row 0, T3 row 1, T0 row 2, T1 row 3.
        const uint32_t e0 = tlook<TAB>(w[c], lb[2], 0);
        const uint32_t e1 = tlook<TAB>(w[(c + 1) & 3], lb[3], 1);
        const uint32_t e2 = tlook<TAB>(w[(c + 2) & 3], lb[0], 2);
        const uint32_t e3 = tlook<TAB>(w[(c + 3) & 3], lb[1], 3);
        const uint32_t u = __byte_perm(e0, e1, 0x0050u);
        const uint32_t v = __byte_perm(e2, e3, 0x7200u);
        n[c] = __byte_perm(u, v, 0x7610u) ^ rk[40 + c];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        w[c] = n[c];
    }
}

// Full encryption of state w (already xored with round key 0).
template <uint32_t TAB>
__device__ __forceinline__ void aes_rounds_smem(uint32_t w[4], const uint32_t* rk, const uint32_t lb[4])
{
    aes_rounds_from<TAB, 1>(w, rk, lb);
}

// Counter-mode round caching. A thread's counters are c0 + 256*k (or + 512*k),
// so counter byte 15 is fixed and bytes 12..13 change only on a carry out of
// byte 14. Round 1 then has a single varying lookup (column 1, T2 of state
// byte 14) and round 2 one varying lookup per column (all from column 1).
// The cache holds the constant parts for the current value of ctr >> 16.
struct CtrCache {
    uint32_t epoch;  // ctr >> 16 the cache was built for
    uint32_t k1;     // round-1 column 1 without T2[state byte 14]
    uint32_t l[4];   // round-2 columns without their column-1 term
};

// s012 = IV words xor round key 0 (state columns 0..2 before round 1).
template <uint32_t TAB>
__device__ __forceinline__ void ctr_cache_build(CtrCache& cc, uint32_t ctr, const uint32_t s012[3],
                                                const uint32_t* rk, const uint32_t lb[4])
{
    const uint32_t s0 = s012[0], s1 = s012[1], s2 = s012[2];
    const uint32_t s3 = bswap32(ctr) ^ rk[3];
    const uint32_t n0 = tlook<TAB>(s0, lb[0], 0) ^ tlook<TAB>(s1, lb[1], 1) ^ tlook<TAB>(s2, lb[2], 2) ^
                        tlook<TAB>(s3, lb[3], 3) ^ rk[4];
    const uint32_t n2 = tlook<TAB>(s2, lb[0], 0) ^ tlook<TAB>(s3, lb[1], 1) ^ tlook<TAB>(s0, lb[2], 2) ^
                        tlook<TAB>(s1, lb[3], 3) ^ rk[6];
    const uint32_t n3 = tlook<TAB>(s3, lb[0], 0) ^ tlook<TAB>(s0, lb[1], 1) ^ tlook<TAB>(s1, lb[2], 2) ^
                        tlook<TAB>(s2, lb[3], 3) ^ rk[7];
    cc.k1 = tlook<TAB>(s1, lb[0], 0) ^ tlook<TAB>(s2, lb[1], 1) ^ tlook<TAB>(s0, lb[3], 3) ^ rk[5];
    cc.l[0] = tlook<TAB>(n0, lb[0], 0) ^ tlook<TAB>(n2, lb[2], 2) ^ tlook<TAB>(n3, lb[3], 3) ^ rk[8];
    cc.l[1] = tlook<TAB>(n2, lb[1], 1) ^ tlook<TAB>(n3, lb[2], 2) ^ tlook<TAB>(n0, lb[3], 3) ^ rk[9];
    cc.l[2] = tlook<TAB>(n2, lb[0], 0) ^ tlook<TAB>(n3, lb[1], 1) ^ tlook<TAB>(n0, lb[2], 2) ^ rk[10];
    cc.l[3] = tlook<TAB>(n3, lb[0], 0) ^ tlook<TAB>(n0, lb[1], 1) ^ tlook<TAB>(n2, lb[3], 3) ^ rk[11];
    cc.epoch = ctr >> 16;
}

// Rounds 1..2 of E_K(IV || BE32(ctr)) from the cache; rk3x = bswap32(rk[3]).
template <uint32_t TAB>
__device__ __forceinline__ void ctr_rounds12(uint32_t w[4], uint32_t ctr, const CtrCache& cc, uint32_t rk3x,
                                             const uint32_t lb[4])
{
    // state byte 14 = counter byte 14 ^ key byte = byte 1 of (ctr ^ bswap(rk3))
    const uint32_t n1 = cc.k1 ^ lds32<TAB>(__byte_perm(ctr ^ rk3x, lb[2], 0x7614u));
    w[0] = cc.l[0] ^ tlook<TAB>(n1, lb[1], 1);
    w[1] = cc.l[1] ^ tlook<TAB>(n1, lb[0], 0);
    w[2] = cc.l[2] ^ tlook<TAB>(n1, lb[3], 3);
    w[3] = cc.l[3] ^ tlook<TAB>(n1, lb[2], 2);
}

// Two keystream blocks for counters c0 < c1. Fast path (both in the cached
// epoch): rounds 1-2 from the cache, rounds 3-10 of both blocks in one basic
// block so their lookups interleave. Otherwise (first use, a carry into byte
// 13, or counters of padding slots): full AES on both, cache rebuilt for c1.
template <uint32_t TAB>
__device__ __forceinline__ void aes_ctr2_cached(uint32_t x[4], uint32_t y[4], uint32_t c0, uint32_t c1,
                                                CtrCache& cc, const uint32_t s012[3], uint32_t rk3x,
                                                const uint32_t* rk, const uint32_t lb[4])
{
    if ((c0 >> 16) == cc.epoch && (c1 >> 16) == cc.epoch) {
        ctr_rounds12<TAB>(x, c0, cc, rk3x, lb);
        ctr_rounds12<TAB>(y, c1, cc, rk3x, lb);
        aes_rounds_from<TAB, 3>(x, rk, lb);
        aes_rounds_from<TAB, 3>(y, rk, lb);
    } else {
        x[0] = y[0] = s012[0];
        x[1] = y[1] = s012[1];
        x[2] = y[2] = s012[2];
        x[3] = bswap32(c0) ^ rk[3];
        y[3] = bswap32(c1) ^ rk[3];
        aes_rounds_from<TAB, 1>(x, rk, lb);
        aes_rounds_from<TAB, 1>(y, rk, lb);
        ctr_cache_build<TAB>(cc, c1, s012, rk, lb);
    }
}

// Counter-mode round caching for one warp's rows: lane l of row r takes
// counter c0 + 32 r + l, so counter bytes 12..14 change only on a carry out of
// byte 15. Within an epoch (ctr >> 8) round 1 has a single varying lookup
// (column 0, T3 of state byte 15) and round 2 one varying lookup per column
// (all from column 0): 5 lookups instead of 32.
struct WarpCtrCache {
    uint32_t epoch;  // ctr >> 8 the cache was built for
    uint32_t k0;     // round-1 column 0 without T3[state byte 15]
    uint32_t l[4];   // round-2 columns without their column-0 term
};

// Builds the cache for the epoch of ctr (its byte 15 is not used).
template <uint32_t TAB>
__device__ __forceinline__ void warp_ctr_cache_build(WarpCtrCache& cc, uint32_t ctr, const uint32_t s012[3],
                                                     const uint32_t* rk, const uint32_t lb[4])
{
    const uint32_t s0 = s012[0], s1 = s012[1], s2 = s012[2];
    const uint32_t s3 = bswap32(ctr) ^ rk[3];
    const uint32_t n1 = tlook<TAB>(s1, lb[0], 0) ^ tlook<TAB>(s2, lb[1], 1) ^ tlook<TAB>(s3, lb[2], 2) ^
                        tlook<TAB>(s0, lb[3], 3) ^ rk[5];
    const uint32_t n2 = tlook<TAB>(s2, lb[0], 0) ^ tlook<TAB>(s3, lb[1], 1) ^ tlook<TAB>(s0, lb[2], 2) ^
                        tlook<TAB>(s1, lb[3], 3) ^ rk[6];
    const uint32_t n3 = tlook<TAB>(s3, lb[0], 0) ^ tlook<TAB>(s0, lb[1], 1) ^ tlook<TAB>(s1, lb[2], 2) ^
                        tlook<TAB>(s2, lb[3], 3) ^ rk[7];
    cc.k0 = tlook<TAB>(s0, lb[0], 0) ^ tlook<TAB>(s1, lb[1], 1) ^ tlook<TAB>(s2, lb[2], 2) ^ rk[4];
    cc.l[0] = tlook<TAB>(n1, lb[1], 1) ^ tlook<TAB>(n2, lb[2], 2) ^ tlook<TAB>(n3, lb[3], 3) ^ rk[8];
    cc.l[1] = tlook<TAB>(n1, lb[0], 0) ^ tlook<TAB>(n2, lb[1], 1) ^ tlook<TAB>(n3, lb[2], 2) ^ rk[9];
    cc.l[2] = tlook<TAB>(n2, lb[0], 0) ^ tlook<TAB>(n3, lb[1], 1) ^ tlook<TAB>(n1, lb[3], 3) ^ rk[10];
    cc.l[3] = tlook<TAB>(n3, lb[0], 0) ^ tlook<TAB>(n1, lb[2], 2) ^ tlook<TAB>(n2, lb[3], 3) ^ rk[11];
    cc.epoch = ctr >> 8;
}

// Keystream block E_K(IV || BE32(ctr)) for one warp row (every lane calls it
// with its own counter; the counters of a row are consecutive). When every
// lane's counter is in the cached epoch: rounds 1-2 from the cache. Otherwise
// the whole warp runs the full cipher and rebuilds the cache for the next
// row's counters (ctr + 32), so a row crossing an epoch boundary costs one
// slow row and no divergence.
template <uint32_t TAB>
__device__ __forceinline__ void warp_ctr_keystream(uint32_t x[4], uint32_t ctr, WarpCtrCache& cc,
                                                   const uint32_t s012[3], const uint32_t* rk, const uint32_t lb[4])
{
    if (__all_sync(0xffffffffu, (ctr >> 8) == cc.epoch)) {
        const uint32_t n0 = cc.k0 ^ tlook<TAB>(bswap32(ctr) ^ rk[3], lb[3], 3);
        x[0] = cc.l[0] ^ tlook<TAB>(n0, lb[0], 0);
        x[1] = cc.l[1] ^ tlook<TAB>(n0, lb[3], 3);
        x[2] = cc.l[2] ^ tlook<TAB>(n0, lb[2], 2);
        x[3] = cc.l[3] ^ tlook<TAB>(n0, lb[1], 1);
        aes_rounds_from<TAB, 3>(x, rk, lb);
    } else {
        x[0] = s012[0];
        x[1] = s012[1];
        x[2] = s012[2];
        x[3] = bswap32(ctr) ^ rk[3];
        aes_rounds_from<TAB, 1>(x, rk, lb);
        warp_ctr_cache_build<TAB>(cc, ctr + 32u, s012, rk, lb);
    }
}

// Same cipher reading the compact T-tables from global memory (one-off blocks).
// GMEM: T is global memory, read through the read-only path; otherwise T
// is a copy of the compact tables in shared memory.
template <bool GMEM>
__device__ inline uint4 aes_encrypt_compact(const uint32_t* T, const uint32_t* rk, uint4 in)
{
    auto ld = [T](uint32_t i) __attribute__((always_inline)) { return GMEM ? __ldg(T + i) : T[i]; };
    uint32_t w[4] = {in.x ^ rk[0], in.y ^ rk[1], in.z ^ rk[2], in.w ^ rk[3]};
    for (int r = 1; r < 10; ++r) {
        uint32_t n[4];
        for (int c = 0; c < 4; ++c) {
            n[c] = ld(w[c] & 0xffu) ^ ld(256 + ((w[(c + 1) & 3] >> 8) & 0xffu)) ^
                   ld(512 + ((w[(c + 2) & 3] >> 16) & 0xffu)) ^ ld(768 + (w[(c + 3) & 3] >> 24)) ^ rk[4 * r + c];
        }
        for (int c = 0; c < 4; ++c) {
            w[c] = n[c];
        }
    }
    uint32_t n[4];
    for (int c = 0; c < 4; ++c) {
        const uint32_t e0 = ld(512 + (w[c] & 0xffu));
        const uint32_t e1 = ld(768 + ((w[(c + 1) & 3] >> 8) & 0xffu));
        const uint32_t e2 = ld((w[(c + 2) & 3] >> 16) & 0xffu);
        const uint32_t e3 = ld(256 + (w[(c + 3) & 3] >> 24));
        n[c] = __byte_perm(__byte_perm(e0, e1, 0x0050u), __byte_perm(e2, e3, 0x7200u), 0x7610u) ^
               rk[40 + c];
    }
    return make_uint4(n[0], n[1], n[2], n[3]);
}

__device__ inline uint4 aes_encrypt_gmem(const uint32_t* T, const uint32_t* rk, uint4 in)
{
    return aes_encrypt_compact<true>(T, rk, in);
}

// Fill the 128 KiB replicated T-table region from the compact global tables.
// Table fills run in every CTA's prologue, before any row can start. Each
// thread issues all of its global loads before its first shared store, so the
// fill costs one memory round trip rather than one per entry. Every kernel
// that fills has blockDim.x >= kFillMinThreads.
constexpr int kFillMinThreads = 512;

__device__ __forceinline__ void fill_aes_smem(uint8_t* tab, const uint32_t* T)
{
    constexpr int kN = 8192;
    constexpr int kPer = (kN + kFillMinThreads - 1) / kFillMinThreads;
    uint32_t t[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = static_cast<int>(threadIdx.x + k * blockDim.x);
        t[k] = i < kN ? __ldg(T + (i >> 11) * 256 + ((i >> 3) & 255)) : 0u;
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = static_cast<int>(threadIdx.x + k * blockDim.x);
        if (i < kN) {
            const int tk = i >> 11;
            const int x = (i >> 3) & 255;
            const int q = i & 7;
            const uint32_t off = (static_cast<uint32_t>(tk >> 1) << 16) | (static_cast<uint32_t>(x) << 8) |
                                 (static_cast<uint32_t>(tk & 1) << 7) | (static_cast<uint32_t>(q) << 4);
            *reinterpret_cast<uint4*>(tab + off) = make_uint4(t[k], t[k], t[k], t[k]);
        }
    }
}

// Copies N 16-byte entries from global to shared memory (prologue fills).
template <int N>
__device__ __forceinline__ void fill_smem(uint4* dst, const uint4* src)
{
    constexpr int kPer = (N + kFillMinThreads - 1) / kFillMinThreads;
    uint4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = static_cast<int>(threadIdx.x + k * blockDim.x);
        v[k] = i < N ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = static_cast<int>(threadIdx.x + k * blockDim.x);
        if (i < N) {
            dst[i] = v[k];
        }
    }
}

__device__ __forceinline__ void aes_lane_bases(uint32_t lb[4], int lane)
{
    const uint32_t l4 = static_cast<uint32_t>(lane) << 2;
    lb[0] = l4;
    lb[1] = 0x80u | l4;
    lb[2] = 0x10000u | l4;
    lb[3] = 0x10080u | l4;
}

// ---------------------------------------------------------------- GHASH

// Fill the 64 KiB replicated GHASH region from a compact 4-bit table.
__device__ __forceinline__ void fill_gh_smem(uint8_t* gh, const uint4* compact)
{
    constexpr int kN = 4096;
    constexpr int kPer = (kN + kFillMinThreads - 1) / kFillMinThreads;
    uint4 e[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = static_cast<int>(threadIdx.x + k * blockDim.x);
        const int row = i >> 4;
        e[k] = i < kN ? __ldg(compact + (2 * (row >> 4) + ((i >> 3) & 1)) * 16 + (row & 15))
                      : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = static_cast<int>(threadIdx.x + k * blockDim.x);
        if (i < kN) {
            *reinterpret_cast<uint4*>(gh + i * 16) = e[k];
        }
    }
}

// x * M using the replicated shared table of M at dynamic offset GH
// (32 LDS.128, no bank conflicts).
template <uint32_t GH>
__device__ __forceinline__ uint4 gh_mul_rep(uint4 x, uint32_t lb_lo, uint32_t lb_hi)
{
    uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t xw = word_of(x, w);
        const uint32_t tag = 0x30201000u + 0x40404040u * static_cast<uint32_t>(w);
        const uint32_t lo = (xw & 0x0f0f0f0fu) | tag;
        const uint32_t hi = ((xw >> 4) & 0x0f0f0f0fu) | tag;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t sel = 0x7604u | (static_cast<uint32_t>(k) << 4);
            const uint4 e = lds128<GH>(__byte_perm(lo, lb_lo, sel));
            const uint4 f = lds128<GH>(__byte_perm(hi, lb_hi, sel));
            a0 ^= e.x ^ f.x;
            a1 ^= e.y ^ f.y;
            a2 ^= e.z ^ f.z;
            a3 ^= e.w ^ f.w;
        }
    }
    return make_uint4(a0, a1, a2, a3);
}

// Fill the replicated window table region (kGh5RepBytes at gh) from its
// compact table: 16-byte slot i holds compact entry i >> 3.
__device__ __forceinline__ void fill_gh5_smem(uint8_t* gh, const uint4* compact)
{
    constexpr int kN = kGh5RepBytes / 16;
    constexpr int kBatch = 4;  // loads in flight per thread
    for (int i0 = static_cast<int>(threadIdx.x); i0 < kN; i0 += kBatch * static_cast<int>(blockDim.x)) {
        uint4 e[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            const int i = i0 + k * static_cast<int>(blockDim.x);
            e[k] = i < kN ? __ldg(compact + (i >> 3)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < kBatch; ++k) {
            const int i = i0 + k * static_cast<int>(blockDim.x);
            if (i < kN) {
                reinterpret_cast<uint4*>(gh)[i] = e[k];
            }
        }
    }
}

// One group of gh_mul_rep5: XOR M's entry for field G of w into (a0..a3).
// The field's shift, the mask and the replica offset are issued with the
// load in one asm statement (the shift as gh5_field_at7 does it), so the
// addresses are formed one group at a time.
template <uint32_t GH, int G>
__device__ __forceinline__ void gh5_acc(const uint32_t (&w)[4], uint32_t lb, uint32_t& a0, uint32_t& a1, uint32_t& a2,
                                        uint32_t& a3)
{
    constexpr int r0 = kGhW * G;
    constexpr int wi = r0 >> 5;
    constexpr int sh = r0 & 31;
    constexpr uint32_t imm = kSmemLayoutBase + GH + static_cast<uint32_t>(G) * kGh5GroupStride;
    constexpr uint32_t mask = kGh5Mask7;
    uint4 e;
    if constexpr (sh < 7) {
        asm volatile(
            "{\n\t.reg .b32 t;\n\tshl.b32 t, %4, %5;\n\tand.b32 t, t, %8;\n\tor.b32 t, t, %6;\n\t"
            "ld.shared.v4.u32 {%0, %1, %2, %3}, [t+%7];\n\t}"
            : "=r"(e.x), "=r"(e.y), "=r"(e.z), "=r"(e.w)
            : "r"(w[wi]), "n"(7 - sh), "r"(lb), "n"(imm), "n"(mask));
    } else if constexpr (sh + kGhW <= 32 || wi == 3) {
        asm volatile(
            "{\n\t.reg .b32 t;\n\tshr.b32 t, %4, %5;\n\tand.b32 t, t, %8;\n\tor.b32 t, t, %6;\n\t"
            "ld.shared.v4.u32 {%0, %1, %2, %3}, [t+%7];\n\t}"
            : "=r"(e.x), "=r"(e.y), "=r"(e.z), "=r"(e.w)
            : "r"(w[wi]), "n"(sh - 7), "r"(lb), "n"(imm), "n"(mask));
    } else {
        asm volatile(
            "{\n\t.reg .b32 t;\n\tshf.r.clamp.b32 t, %4, %5, %6;\n\tand.b32 t, t, %9;\n\tor.b32 t, t, %7;\n\t"
            "ld.shared.v4.u32 {%0, %1, %2, %3}, [t+%8];\n\t}"
            : "=r"(e.x), "=r"(e.y), "=r"(e.z), "=r"(e.w)
            : "r"(w[wi]), "r"(w[wi + 1]), "n"(sh - 7), "r"(lb), "n"(imm), "n"(mask));
    }
    a0 ^= e.x;
    a1 ^= e.y;
    a2 ^= e.z;
    a3 ^= e.w;
}

// Groups 2P and 2P+1 of gh_mul_rep5, XORed together before the accumulator.
template <uint32_t GH, int P>
__device__ __forceinline__ void gh5_acc_pair(const uint32_t (&w)[4], uint32_t lb, uint32_t& a0, uint32_t& a1,
                                             uint32_t& a2, uint32_t& a3)
{
    uint32_t e0 = 0, e1 = 0, e2 = 0, e3 = 0;
    gh5_acc<GH, 2 * P>(w, lb, e0, e1, e2, e3);
    gh5_acc<GH, 2 * P + 1>(w, lb, e0, e1, e2, e3);
    a0 ^= e0;
    a1 ^= e1;
    a2 ^= e2;
    a3 ^= e3;
}

template <uint32_t GH, int... P>
__device__ __forceinline__ uint4 gh5_mul_groups(const uint32_t (&w)[4], uint32_t lb, std::integer_sequence<int, P...>)
{
    uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    (gh5_acc_pair<GH, P>(w, lb, a0, a1, a2, a3), ...);
    return make_uint4(a0, a1, a2, a3);
}

// x * M using the replicated kGhW-bit-window table of M at dynamic offset GH
// (kGh5Groups LDS.128, no bank conflicts; lb = (lane & 7) << 4 picks the replica).
template <uint32_t GH>
__device__ __forceinline__ uint4 gh_mul_rep5(uint4 x, uint32_t lb)
{
    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
    static_assert(kGh5Groups % 2 == 0, "groups are taken in pairs");
    return gh5_mul_groups<GH>(w, lb, std::make_integer_sequence<int, kGh5Groups / 2>{});
}

// x * M using a compact (non-replicated) table, shared or global memory.
__device__ __forceinline__ uint4 gh_mul_compact(uint4 x, const uint4* tab)
{
    uint4 acc = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint32_t b = byte_of(x, j);
        acc = xor4(acc, tab[(2 * j) * 16 + (b & 15u)]);
        acc = xor4(acc, tab[(2 * j + 1) * 16 + (b >> 4)]);
    }
    return acc;
}

// R independent GHASH Horner chains per thread: chain k takes the thread's
// rows r = k (mod R) with multiplier M = H^(R*T), so the R multiplies of an
// iteration do not wait on one another (only their final XOR waits for the
// row's ciphertext).
template <int R>
struct Chains {
    uint4 q[R];
};

// Push block c of row r into chain r mod R (k known only at run time).
template <uint32_t GH, int R>
__device__ __forceinline__ void chain_push_dyn(Chains<R>& ch, int k, uint4 c, uint32_t lb_lo, uint32_t lb_hi)
{
    uint4 v = ch.q[0];
#pragma unroll
    for (int j = 1; j < R; ++j) {
        if (k == j) {
            v = ch.q[j];
        }
    }
    v = xor4(gh_mul_rep<GH>(v, lb_lo, lb_hi), c);
#pragma unroll
    for (int j = 0; j < R; ++j) {
        if (k == j) {
            ch.q[j] = v;
        }
    }
}

// chain_push_dyn with the replicated window table of M at GH.
template <uint32_t GH, int R>
__device__ __forceinline__ void chain_push_dyn5(Chains<R>& ch, int k, uint4 c, uint32_t lb)
{
    uint4 v = ch.q[0];
#pragma unroll
    for (int j = 1; j < R; ++j) {
        if (k == j) {
            v = ch.q[j];
        }
    }
    v = xor4(gh_mul_rep5<GH>(v, lb), c);
#pragma unroll
    for (int j = 0; j < R; ++j) {
        if (k == j) {
            ch.q[j] = v;
        }
    }
}

// The thread's share over its J rows, sum_r X_r H^(T (J-1-r)), from the R
// chains: chain k's last row is J-1-((J-1-k) mod R), so
//   Q = sum_k q_k H^(T ((J-1-k) mod R)),
// evaluated by Horner with H^T (compact table ht, read through L1).
template <int R>
__device__ __forceinline__ uint4 chains_combine(const Chains<R>& ch, int64_t J, const uint4* ht)
{
    uint4 acc = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int d = R - 1; d >= 0; --d) {
        const int k = static_cast<int>((((J - 1 - d) % R) + R) % R);
        uint4 v = ch.q[0];
#pragma unroll
        for (int j = 1; j < R; ++j) {
            if (k == j) {
                v = ch.q[j];
            }
        }
        acc = (d == R - 1) ? v : xor4(gh_mul_compact(acc, ht), v);
    }
    return acc;
}

// Warp-parallel x * M with a compact global table: lane p looks up nibble
// position p, then a butterfly xor leaves the product in every lane.
__device__ __forceinline__ uint4 warp_gh_mul_global(uint4 x, const uint4* tab, int lane)
{
    const int j = lane >> 1;
    const uint32_t b = byte_of(x, j);
    const uint32_t v = (lane & 1) ? (b >> 4) : (b & 15u);
    uint4 e = __ldg(tab + lane * 16 + v);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        e.x ^= __shfl_xor_sync(0xffffffffu, e.x, o);
        e.y ^= __shfl_xor_sync(0xffffffffu, e.y, o);
        e.z ^= __shfl_xor_sync(0xffffffffu, e.z, o);
        e.w ^= __shfl_xor_sync(0xffffffffu, e.w, o);
    }
    return e;
}

// Power warp, part 1: H^d (raw bytes) from the H^(2^k) tables.
__device__ inline uint4 warp_h_pow(const uint4* pow2, unsigned long long d, int lane)
{
    uint4 m = make_uint4(0x80u, 0, 0, 0);  // identity: bit 0 of byte 0
    int k = 0;
    while (d) {
        if (d & 1ull) {
            m = warp_gh_mul_global(m, pow2 + static_cast<size_t>(k) * 512, lane);
        }
        d >>= 1;
        ++k;
    }
    return m;
}

// 128-bit shifts of (hi, lo) (hi = coefficients x^0..x^63, MSB first) by
// 0 <= s < 128 bits; "right" moves toward higher powers of x.
__device__ __forceinline__ void shr128(unsigned long long& hi, unsigned long long& lo, int s)
{
    if (s >= 64) {
        lo = hi >> (s - 64);
        hi = 0;
    } else if (s > 0) {
        lo = (lo >> s) | (hi << (64 - s));
        hi >>= s;
    }
}

__device__ __forceinline__ void shl128(unsigned long long& hi, unsigned long long& lo, int s)
{
    if (s >= 64) {
        hi = lo << (s - 64);
        lo = 0;
    } else if (s > 0) {
        hi = (hi << s) | (lo >> (64 - s));
        lo <<= s;
    }
}

// (hi, lo) <- (hi, lo) * x^0 + x^1 + x^2 + x^7 applied to an element of degree
// < 121 (no overflow): the reduction polynomial of x^128 in GF(2^128).
__device__ __forceinline__ void mul_r(unsigned long long& hi, unsigned long long& lo)
{
    unsigned long long h1 = hi, l1 = lo, h2 = hi, l2 = lo, h7 = hi, l7 = lo;
    shr128(h1, l1, 1);
    shr128(h2, l2, 2);
    shr128(h7, l7, 7);
    hi ^= h1 ^ h2 ^ h7;
    lo ^= l1 ^ l2 ^ l7;
}

// V * x^k for 0 <= k < 128 without a loop: shift, then fold the k overflow
// bits back with x^128 = 1 + x + x^2 + x^7 (twice: the second overflow,
// from the x^2 and x^7 terms when k > 121, has degree < 7).
__device__ inline void gf_mul_xk(unsigned long long& hi, unsigned long long& lo, int k)
{
    if (k == 0) {
        return;
    }
    unsigned long long oh = hi, ol = lo;  // overflow: the low k bits moved to the top
    shl128(oh, ol, 128 - k);
    shr128(hi, lo, k);
    // second-level overflow of O*(x^2 + x^7): the low 2 and 7 bits of O
    unsigned long long ph = oh, pl = ol, qh = oh, ql = ol;
    shl128(ph, pl, 126);
    shl128(qh, ql, 121);
    unsigned long long o2h = ph ^ qh, o2l = pl ^ ql;
    // O * (1 + x + x^2 + x^7), keeping only the part that stays below x^128
    unsigned long long rh = oh, rl = ol;
    {
        unsigned long long h1 = oh, l1 = ol, h2 = oh, l2 = ol, h7 = oh, l7 = ol;
        shr128(h1, l1, 1);
        shr128(h2, l2, 2);
        shr128(h7, l7, 7);
        rh ^= h1 ^ h2 ^ h7;
        rl ^= l1 ^ l2 ^ l7;
    }
    mul_r(o2h, o2l);
    hi ^= rh ^ o2h;
    lo ^= rl ^ o2l;
}

// Power warp, part 2: lane p keeps U_p = M * x^(4p) for the final multiply.
__device__ inline void warp_lane_basis(uint4 m_raw, int lane, unsigned long long& uhi,
                                       unsigned long long& ulo)
{
    raw_to_be(m_raw, uhi, ulo);
    gf_mul_xk(uhi, ulo, 4 * lane);
}

// Power warp, part 3: F * M where lane p holds U_p = M * x^(4p); result
// (big-endian halves) in every lane.
__device__ inline void warp_generic_mul(uint4 f_raw, unsigned long long uhi, unsigned long long ulo,
                                        int lane, unsigned long long& rhi, unsigned long long& rlo)
{
    // bits 4p..4p+3 of F (SP 800-38D order: MSB of byte 0 first)
    const uint32_t b = byte_of(f_raw, lane >> 1);
    const uint32_t nib = (lane & 1) ? (b & 15u) : (b >> 4);
    unsigned long long ahi = 0, alo = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const unsigned long long m = 0ull - static_cast<unsigned long long>((nib >> (3 - k)) & 1u);
        ahi ^= uhi & m;
        alo ^= ulo & m;
        gf_mul_x(uhi, ulo);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        ahi ^= __shfl_xor_sync(0xffffffffu, ahi, o);
        alo ^= __shfl_xor_sync(0xffffffffu, alo, o);
    }
    rhi = ahi;
    rlo = alo;
}

// H^d (raw bytes) on the integer pipes, for d < 2^32 (larger d: warp_h_pow).
// Lane k loads M_k = H^(2^k) when bit k of d is set (entry 24 of the compact
// table of M is M itself: the identity block has only the high nibble of byte
// 0 set, to 8), so all factors arrive in one memory round trip; the product
// then takes one warp_generic_mul by the lane basis of each further factor.
// warp_h_pow instead waits for one global-table lookup per set bit, which in
// a per-object call of a few rows per tile outlasts the rows.
__device__ inline uint4 warp_h_pow_alu(const uint4* pow2, unsigned long long d, int lane)
{
    if ((d >> 32) != 0ull) {
        return warp_h_pow(pow2, d, lane);
    }
    uint4 mine = make_uint4(0, 0, 0, 0);
    if ((d >> lane) & 1ull) {
        mine = __ldg(pow2 + static_cast<size_t>(lane) * 512 + 24);
    }
    uint4 m = make_uint4(0x80u, 0, 0, 0);  // identity
    bool first = true;
    while (d) {
        const int k = __ffsll(static_cast<long long>(d)) - 1;
        d &= d - 1ull;
        const uint4 f = shfl4(mine, k);
        if (first) {
            m = f;
            first = false;
            continue;
        }
        unsigned long long uhi, ulo, rhi, rlo;
        warp_lane_basis(f, lane, uhi, ulo);
        warp_generic_mul(m, uhi, ulo, lane, rhi, rlo);
        m = be_to_raw(rhi, rlo);
    }
    return m;
}

// Power-warp epilogue of seal/open GHASH: scale the CTA's fold by H^(d_c)
// (lane p holds U_p = H^(d_c) x^(4p)), XOR it into the call's slot and take
// a ticket. Returns true in every lane of the last CTA to arrive, with the
// full sum S (before the length block) in (shi, slo); that CTA also resets
// the slot for the next call. No CTA waits on another.
__device__ inline bool cta_accumulate(Slot* slot, uint4 fold, unsigned long long uhi, unsigned long long ulo,
                                      int lane, uint32_t grid, unsigned long long& shi, unsigned long long& slo)
{
    unsigned long long rhi, rlo;
    warp_generic_mul(fold, uhi, ulo, lane, rhi, rlo);
    unsigned int ticket = 0;
    if (lane == 0) {
        atomicXor(&slot->acc_hi, rhi);
        atomicXor(&slot->acc_lo, rlo);
        __threadfence();
        ticket = atomicAdd(&slot->ticket, 1u);
    }
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != grid - 1) {
        return false;
    }
    __threadfence();
    unsigned long long h = 0, l = 0;
    if (lane == 0) {
        h = atomicXor(&slot->acc_hi, 0ull);
        l = atomicXor(&slot->acc_lo, 0ull);
        slot->acc_hi = 0;
        slot->acc_lo = 0;
        slot->ticket = 0;
    }
    shi = __shfl_sync(0xffffffffu, h, 0);
    slo = __shfl_sync(0xffffffffu, l, 0);
    return true;
}

// Fold the kHornerThreads partials in shared memory, levels [first, last):
// after level l the entry at index p * 2^(l+1) holds left * H^(2^l) + right.
// Levels l < NSMEM read the compact table of H^(2^l) staged in shared memory
// at smem_tabs + 512 (l - first); the rest read it from global memory
// (pow2 + 512 l) through L1. A zero left operand (rows the object does not
// reach) skips its multiply.
template <int NSMEM>
__device__ __forceinline__ void fold_partials(uint4* part, const uint4* smem_tabs, const uint4* pow2,
                                              int first = 0, int last = kFoldLevels)
{
#pragma unroll 1
    for (int l = first; l < last; ++l) {
        const int pairs = kHornerThreads >> (l + 1);
        const int t = threadIdx.x;
        if (t < pairs) {
            const int left = t << (l + 1);
            const uint4 x = part[left];
            uint4 m = make_uint4(0, 0, 0, 0);
            if ((x.x | x.y | x.z | x.w) != 0u) {
                m = gh_mul_compact(x, l < NSMEM ? smem_tabs + (l - first) * 512 : pow2 + l * 512);
            }
            part[left] = xor4(m, part[left + (1 << l)]);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------- byte helpers

__device__ __forceinline__ void store_bytes(uint8_t* dst, uint4 v, int lo, int hi)
{
    for (int b = lo; b < hi; ++b) {
        dst[b] = static_cast<uint8_t>(byte_of(v, b));
    }
}

__device__ __forceinline__ uint4 load_bytes(const uint8_t* src, int n)
{
    uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
    for (int b = 0; b < n; ++b) {
        const uint32_t v = static_cast<uint32_t>(src[b]) << (8 * (b & 3));
        if (b < 4) {
            w0 |= v;
        } else if (b < 8) {
            w1 |= v;
        } else if (b < 12) {
            w2 |= v;
        } else {
            w3 |= v;
        }
    }
    return make_uint4(w0, w1, w2, w3);
}

__device__ __forceinline__ uint4 mask_bytes(uint4 v, int n)
{
    // keep bytes [0, n), zero the rest (0 <= n <= 16)
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int keep = n - 4 * k;
        const uint32_t m = keep >= 4 ? 0xffffffffu : keep <= 0 ? 0u : ((1u << (8 * keep)) - 1u);
        w[k] &= m;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// Bytes of block i of a P-byte object: 16 for i < P/16, the remainder for the
// last partial block, 0 outside [0, n).
__device__ __forceinline__ int block_bytes(int64_t i, uint64_t P)
{
    if (i < 0) {
        return 0;
    }
    const uint64_t off = static_cast<uint64_t>(i) * 16u;
    if (off >= P) {
        return 0;
    }
    const uint64_t rem = P - off;
    return rem >= 16 ? 16 : static_cast<int>(rem);
}

// Block i of a plaintext buffer (zero-padded; zero outside the object).
template <bool ALIGNED>
__device__ __forceinline__ uint4 load_pt_block(const uint8_t* src, int64_t i, uint64_t P)
{
    const int nb = block_bytes(i, P);
    const uint8_t* p = src + static_cast<uint64_t>(i) * 16u;
    if (ALIGNED && nb == 16) {
        return __ldg(reinterpret_cast<const uint4*>(p));
    }
    if (nb == 0) {
        return make_uint4(0, 0, 0, 0);
    }
    return load_bytes(p, nb);
}

// Block i of the ciphertext at frame + 13, in two steps. ct_prefetch issues the
// loads: LQ = word part of (frame + 13) & 15 (4 = aligned); a lane reads the
// two aligned 16-B chunks covering its block when both lie inside the frame
// buffer. ct_finish applies the funnel (byte part in the PRMT selector fsel),
// or falls back to byte loads for partial / edge blocks; zero outside the
// object. Issuing the prefetch one iteration ahead hides the load latency.
struct CtRaw {
    uint4 d;
    uint4 e;
    bool fast;
};

template <int LQ>
__device__ __forceinline__ CtRaw ct_prefetch(const uint8_t* frame, uint64_t frame_len, int64_t i, uint64_t P)
{
    CtRaw r{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), false};
    if (block_bytes(i, P) == 16) {
        const uint8_t* ct = frame + 13 + static_cast<uint64_t>(i) * 16u;
        if (LQ == 4) {
            r.d = *reinterpret_cast<const uint4*>(ct);
            r.fast = true;
        } else {
            const uint8_t* c0 = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(ct) &
                                                                 ~static_cast<uintptr_t>(15));
            if (c0 >= frame && c0 + 32 <= frame + frame_len) {
                r.d = *reinterpret_cast<const uint4*>(c0);
                r.e = *reinterpret_cast<const uint4*>(c0 + 16);
                r.fast = true;
            }
        }
    }
    return r;
}

template <int LQ>
__device__ __forceinline__ uint4 ct_finish(const CtRaw& r, const uint8_t* frame, int64_t i, uint64_t P,
                                           uint32_t fsel)
{
    if (r.fast) {
        if (LQ == 4) {
            return r.d;
        }
        const uint32_t sw[8] = {r.d.x, r.d.y, r.d.z, r.d.w, r.e.x, r.e.y, r.e.z, r.e.w};
        constexpr int q = LQ & 3;
        return make_uint4(funnel(sw[q], sw[q + 1], fsel), funnel(sw[q + 1], sw[q + 2], fsel),
                          funnel(sw[q + 2], sw[q + 3], fsel), funnel(sw[q + 3], sw[q + 4], fsel));
    }
    const int nb = block_bytes(i, P);
    if (nb == 0) {
        return make_uint4(0, 0, 0, 0);
    }
    return load_bytes(frame + 13 + static_cast<uint64_t>(i) * 16u, nb);
}

// Store ciphertext block i (nb valid bytes, nb = 0 for no block) at
// ct + 16 i. SQ = 4: ct is 16-B aligned. SQ = 0..3: ct is misaligned by
// 16 - s (s = 4 SQ + r); lane l writes the aligned chunk at ct + 16 i + s,
// built from its block and lane l+1's block (one shuffle per needed word),
// when both are in this warp and the chunk lies inside [0, P); warp-edge and
// object-edge bytes go out byte-wise. Every lane of the warp must call this.
template <int SQ>
__device__ __forceinline__ void store_ct_block(uint8_t* ct, int64_t i, uint4 c, int nb, uint64_t P,
                                               uint32_t s, uint32_t fsel, int lane)
{
    const uint64_t off = static_cast<uint64_t>(i) * 16u;
    if constexpr (SQ == 4) {
        if (nb == 16) {
            *reinterpret_cast<uint4*>(ct + off) = c;
        } else if (nb > 0) {
            store_bytes(ct + off, c, 0, nb);
        }
        return;
    } else {
    uint32_t nbw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        nbw[k] = k <= (SQ & 3) ? __shfl_down_sync(0xffffffffu, word_of(c, k), 1) : 0u;
    }
    const bool valid = nb > 0;
    const bool full = valid && lane < 31 && off + s + 16 <= P;
    const bool prev_full = valid && lane > 0 && i >= 1 && off + s <= P;
    if (full) {
        const uint32_t sw[8] = {c.x, c.y, c.z, c.w, nbw[0], nbw[1], nbw[2], nbw[3]};
        uint4 o;
        o.x = funnel(sw[(SQ & 3) + 0], sw[(SQ & 3) + 1], fsel);
        o.y = funnel(sw[(SQ & 3) + 1], sw[(SQ & 3) + 2], fsel);
        o.z = funnel(sw[(SQ & 3) + 2], sw[(SQ & 3) + 3], fsel);
        o.w = funnel(sw[(SQ & 3) + 3], sw[(SQ & 3) + 4], fsel);
        *reinterpret_cast<uint4*>(ct + off + s) = o;
    } else if (valid) {
        store_bytes(ct + off, c, static_cast<int>(s), nb);
    }
    if (valid && !prev_full) {
        store_bytes(ct + off, c, 0, nb < static_cast<int>(s) ? nb : static_cast<int>(s));
    }
    }
}

// Bytes [0, n) of v to a 16-byte aligned destination, widest stores first.
__device__ __forceinline__ void store_prefix_aligned(uint8_t* dst, uint4 v, uint32_t n)
{
    uint32_t k = 0;
    if (n & 8u) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(v.x, v.y);
        k = 8;
    }
    if (n & 4u) {
        *reinterpret_cast<uint32_t*>(dst + k) = word_of(v, static_cast<int>(k >> 2));
        k += 4;
    }
    if (n & 2u) {
        const uint32_t w = word_of(v, static_cast<int>(k >> 2));
        *reinterpret_cast<uint16_t*>(dst + k) = static_cast<uint16_t>(w >> (8 * (k & 3u)));
        k += 2;
    }
    if (n & 1u) {
        dst[k] = static_cast<uint8_t>(byte_of(v, static_cast<int>(k)));
    }
}

// Bytes [4q + r, 4q + r + 16) of the 32-byte window (d, e) -- two adjacent
// aligned 16-byte chunks -- for a runtime word offset q (0..3) and byte
// offset r (in fsel = funnel_sel(r)).
__device__ __forceinline__ uint4 window16(uint4 d, uint4 e, uint32_t q, uint32_t fsel)
{
    uint32_t w0 = d.x, w1 = d.y, w2 = d.z, w3 = d.w, w4 = e.x, w5 = e.y;
    if (q & 2u) {
        w0 = w2;
        w1 = w3;
        w2 = w4;
        w3 = w5;
        w4 = e.z;
        w5 = e.w;
    }
    if (q & 1u) {
        w0 = w1;
        w1 = w2;
        w2 = w3;
        w3 = w4;
        w4 = w5;
    }
    return make_uint4(funnel(w0, w1, fsel), funnel(w1, w2, fsel), funnel(w2, w3, fsel), funnel(w3, w4, fsel));
}

// Store of block c at p = dst + 16 i for a row whose 32 lanes all hold full
// blocks inside the object, dst misaligned by 16 - s (s = 4 q + r, 1..15,
// runtime): lanes 0..30 write the aligned chunk at p + s built from their
// block and the next lane's; lane 31 writes the first 16 - s bytes of that
// chunk and lane 0 its block's first s bytes. Every lane of the warp must
// call this.
__device__ __forceinline__ void store_funnel_rt(uint8_t* p, uint4 c, uint32_t s, uint32_t q, uint32_t fsel,
                                                int lane)
{
    const uint4 nb = make_uint4(__shfl_down_sync(0xffffffffu, c.x, 1), __shfl_down_sync(0xffffffffu, c.y, 1),
                                __shfl_down_sync(0xffffffffu, c.z, 1), __shfl_down_sync(0xffffffffu, c.w, 1));
    const uint4 o = window16(c, nb, q, fsel);
    if (lane < 31) {
        *reinterpret_cast<uint4*>(p + s) = o;
    } else {
        store_prefix_aligned(p + s, o, 16u - s);
    }
    if (lane == 0) {
        store_bytes(p, c, 0, static_cast<int>(s));
    }
}

// store_ct_block for a ciphertext pointer misaligned by a runtime 16 - s
// (s = 4 q + r in 1..15, fsel = funnel_sel(r)): same chunk / byte split.
// Every lane of the warp must call this.
__device__ __forceinline__ void store_ct_block_rt(uint8_t* ct, int64_t i, uint4 c, int nb, uint64_t P, uint32_t s,
                                                  uint32_t q, uint32_t fsel, int lane)
{
    const uint64_t off = static_cast<uint64_t>(i) * 16u;
    const uint4 nbv = make_uint4(__shfl_down_sync(0xffffffffu, c.x, 1), __shfl_down_sync(0xffffffffu, c.y, 1),
                                 __shfl_down_sync(0xffffffffu, c.z, 1), __shfl_down_sync(0xffffffffu, c.w, 1));
    const bool valid = nb > 0;
    const bool full = valid && lane < 31 && off + s + 16 <= P;
    const bool prev_full = valid && lane > 0 && i >= 1 && off + s <= P;
    if (full) {
        *reinterpret_cast<uint4*>(ct + off + s) = window16(c, nbv, q, fsel);
    } else if (valid) {
        store_bytes(ct + off, c, static_cast<int>(s), nb);
    }
    if (valid && !prev_full) {
        store_bytes(ct + off, c, 0, nb < static_cast<int>(s) ? nb : static_cast<int>(s));
    }
}

// Ciphertext block i of a frame (zero outside the object) with a runtime
// load class: off = (frame + 13) & 15, q = off >> 2, fsel = funnel_sel(off
// & 3). Full blocks whose two aligned chunks lie inside the frame take two
// vector loads and a funnel; edge blocks take byte loads.
__device__ __forceinline__ uint4 ct_block_rt(const uint8_t* frame, uint64_t frame_len, int64_t i, uint64_t P,
                                             uint32_t off, uint32_t q, uint32_t fsel)
{
    const int nb = block_bytes(i, P);
    if (nb == 0) {
        return make_uint4(0, 0, 0, 0);
    }
    const uint8_t* ct = frame + 13 + static_cast<uint64_t>(i) * 16u;
    if (nb == 16) {
        if (off == 0) {
            return *reinterpret_cast<const uint4*>(ct);
        }
        const uint8_t* c0 = ct - off;
        if (c0 >= frame && c0 + 32 <= frame + frame_len) {
            return window16(*reinterpret_cast<const uint4*>(c0), *reinterpret_cast<const uint4*>(c0 + 16), q, fsel);
        }
    }
    return load_bytes(ct, nb);
}

// Store of ciphertext block i at ctp = ct + 16 i for a row whose 32 lanes all
// hold full blocks inside the object. SQ = 4: ct aligned, one vector store.
// Otherwise lanes 0..30 write the aligned chunk at ctp + s built from their
// block and the next lane's; lane 31 writes the first 16 - s bytes of that
// chunk (its block's tail; the next warp's lane 0 writes the rest) and lane 0
// writes its block's first s bytes. No bounds checks: the caller guarantees
// the row is interior. Every lane of the warp must call this.
template <int SQ>
__device__ __forceinline__ void store_ct_interior(uint8_t* ctp, uint4 c, uint32_t s, uint32_t fsel, int lane)
{
    if constexpr (SQ == 4) {
        *reinterpret_cast<uint4*>(ctp) = c;
    } else {
        uint32_t nbw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            nbw[k] = k <= (SQ & 3) ? __shfl_down_sync(0xffffffffu, word_of(c, k), 1) : 0u;
        }
        const uint32_t sw[8] = {c.x, c.y, c.z, c.w, nbw[0], nbw[1], nbw[2], nbw[3]};
        constexpr int q = SQ & 3;
        uint4 o;
        o.x = funnel(sw[q + 0], sw[q + 1], fsel);
        o.y = funnel(sw[q + 1], sw[q + 2], fsel);
        o.z = funnel(sw[q + 2], sw[q + 3], fsel);
        o.w = funnel(sw[q + 3], sw[q + 4], fsel);
        if (lane < 31) {
            *reinterpret_cast<uint4*>(ctp + s) = o;
        } else {
            store_prefix_aligned(ctp + s, o, 16u - s);
        }
        if (lane == 0) {
            store_bytes(ctp, c, 0, static_cast<int>(s));
        }
    }
}

}  // namespace dev
}  // namespace confkv
