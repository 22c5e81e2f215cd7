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

namespace confkv {
namespace dev {

constexpr int kHornerThreads = 256;                 // GHASH chains per CTA
constexpr int kFoldLevels = 8;                      // log2(kHornerThreads)
constexpr int kPowerWarp = kHornerThreads / 32;     // warp index of the power warp
constexpr int kSealThreads = kHornerThreads + 32;
constexpr int kCtrThreads = 512;

// Shared-memory regions (byte offsets from the dynamic shared base).
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

constexpr uint32_t kSealAes = 0;
constexpr uint32_t kSealGh = kSealAes + kAesBytes;
constexpr uint32_t kSealPart = kSealGh + kGhBytes;
constexpr uint32_t kSealMisc = kSealPart + kPartBytes;
constexpr uint32_t kSealSmem = kSealMisc + 64;

constexpr uint32_t kOpenGh = 0;
constexpr uint32_t kOpenPart = kOpenGh + kGhBytes;
constexpr uint32_t kOpenMisc = kOpenPart + kPartBytes;
constexpr uint32_t kOpenSmem = kOpenMisc + 64;

constexpr uint32_t kCtrSmem = kAesBytes;

// Per-call accumulation slot (32 bytes). The last CTA of a call resets it.
struct Slot {
    unsigned long long acc_hi;
    unsigned long long acc_lo;
    unsigned int ticket;
    unsigned int pad[3];
};

struct KeyTables {
    const uint32_t* aes_t;   // T0..T3, 4 x 256 words
    const uint4* gh_main;    // compact 4-bit table for H^kHornerThreads (512 entries)
    const uint4* gh_pow2;    // compact 4-bit tables for H^(2^k), k = 0..35
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
};

struct CtrArgs {
    const uint8_t* frame;
    uint64_t frame_len;
    uint8_t* dst;
    uint64_t plen;
    uint32_t nblocks;
    uint32_t load_r;
    uint32_t rk[44];
    const uint32_t* aes_t;
    const int* auth_ok;
};

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

// One T-table lookup in the replicated shared-memory tables: index byte m of
// w, table half/lane from lb (byte 0 and byte 2 of lb are passed through).
__device__ __forceinline__ uint32_t tlook(const uint8_t* tab, uint32_t w, uint32_t lb, int m)
{
    const uint32_t off = __byte_perm(w, lb, 0x7604u | (static_cast<uint32_t>(m) << 4));
    return *reinterpret_cast<const uint32_t*>(tab + off);
}

// Encrypt state w (already xored with round key 0) with the shared tables.
__device__ __forceinline__ void aes_rounds_smem(uint32_t w[4], const uint32_t* rk,
                                                const uint8_t* tab, const uint32_t lb[4])
{
#pragma unroll
    for (int r = 1; r < 10; ++r) {
        uint32_t n[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            n[c] = tlook(tab, w[c], lb[0], 0) ^ tlook(tab, w[(c + 1) & 3], lb[1], 1) ^
                   tlook(tab, w[(c + 2) & 3], lb[2], 2) ^ tlook(tab, w[(c + 3) & 3], lb[3], 3) ^
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
        const uint32_t e0 = tlook(tab, w[c], lb[2], 0);
        const uint32_t e1 = tlook(tab, w[(c + 1) & 3], lb[3], 1);
        const uint32_t e2 = tlook(tab, w[(c + 2) & 3], lb[0], 2);
        const uint32_t e3 = tlook(tab, w[(c + 3) & 3], lb[1], 3);
        const uint32_t u = __byte_perm(e0, e1, 0x0050u);
        const uint32_t v = __byte_perm(e2, e3, 0x7200u);
        n[c] = __byte_perm(u, v, 0x7610u) ^ rk[40 + c];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        w[c] = n[c];
    }
}

// Same cipher reading the compact T-tables from global memory (one-off blocks).
__device__ inline uint4 aes_encrypt_gmem(const uint32_t* T, const uint32_t* rk, uint4 in)
{
    uint32_t w[4] = {in.x ^ rk[0], in.y ^ rk[1], in.z ^ rk[2], in.w ^ rk[3]};
    for (int r = 1; r < 10; ++r) {
        uint32_t n[4];
        for (int c = 0; c < 4; ++c) {
            n[c] = __ldg(T + (w[c] & 0xffu)) ^ __ldg(T + 256 + ((w[(c + 1) & 3] >> 8) & 0xffu)) ^
                   __ldg(T + 512 + ((w[(c + 2) & 3] >> 16) & 0xffu)) ^
                   __ldg(T + 768 + (w[(c + 3) & 3] >> 24)) ^ rk[4 * r + c];
        }
        for (int c = 0; c < 4; ++c) {
            w[c] = n[c];
        }
    }
    uint32_t n[4];
    for (int c = 0; c < 4; ++c) {
        const uint32_t e0 = __ldg(T + 512 + (w[c] & 0xffu));
        const uint32_t e1 = __ldg(T + 768 + ((w[(c + 1) & 3] >> 8) & 0xffu));
        const uint32_t e2 = __ldg(T + ((w[(c + 2) & 3] >> 16) & 0xffu));
        const uint32_t e3 = __ldg(T + 256 + (w[(c + 3) & 3] >> 24));
        n[c] = __byte_perm(__byte_perm(e0, e1, 0x0050u), __byte_perm(e2, e3, 0x7200u), 0x7610u) ^
               rk[40 + c];
    }
    return make_uint4(n[0], n[1], n[2], n[3]);
}

// Fill the 128 KiB replicated T-table region from the compact global tables.
__device__ __forceinline__ void fill_aes_smem(uint8_t* tab, const uint32_t* T)
{
    for (int i = threadIdx.x; i < 8192; i += blockDim.x) {
        const int k = i >> 11;
        const int x = (i >> 3) & 255;
        const int q = i & 7;
        const uint32_t t = __ldg(T + k * 256 + x);
        const uint32_t off = (static_cast<uint32_t>(k >> 1) << 16) | (static_cast<uint32_t>(x) << 8) |
                             (static_cast<uint32_t>(k & 1) << 7) | (static_cast<uint32_t>(q) << 4);
        *reinterpret_cast<uint4*>(tab + off) = make_uint4(t, t, t, t);
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
    for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
        const int row = i >> 4;
        const int h = (i >> 3) & 1;
        const int j = row >> 4;
        const int v = row & 15;
        *reinterpret_cast<uint4*>(gh + i * 16) = __ldg(compact + (2 * j + h) * 16 + v);
    }
}

// x * M using the replicated shared table of M (32 LDS.128, no bank conflicts).
__device__ __forceinline__ uint4 gh_mul_rep(uint4 x, const uint8_t* gh, uint32_t lb_lo, uint32_t lb_hi)
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
            const uint4 e = *reinterpret_cast<const uint4*>(gh + __byte_perm(lo, lb_lo, sel));
            const uint4 f = *reinterpret_cast<const uint4*>(gh + __byte_perm(hi, lb_hi, sel));
            a0 ^= e.x ^ f.x;
            a1 ^= e.y ^ f.y;
            a2 ^= e.z ^ f.z;
            a3 ^= e.w ^ f.w;
        }
    }
    return make_uint4(a0, a1, a2, a3);
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

// Power warp, part 2: lane p keeps U_p = M * x^(4p) for the final multiply.
__device__ inline void warp_lane_basis(uint4 m_raw, int lane, unsigned long long& uhi,
                                       unsigned long long& ulo)
{
    raw_to_be(m_raw, uhi, ulo);
    for (int s = 0; s < 4 * lane; ++s) {
        gf_mul_x(uhi, ulo);
    }
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

// Fold the kHornerThreads partials in shared memory: after level l the entry
// at index p * 2^(l+1) holds left * H^(2^l) + right. fold_tabs are the compact
// tables for H^(2^l), l = 0..kFoldLevels-1, staged in shared memory.
__device__ __forceinline__ void fold_partials(uint4* part, const uint4* fold_tabs)
{
#pragma unroll 1
    for (int l = 0; l < kFoldLevels; ++l) {
        const int pairs = kHornerThreads >> (l + 1);
        const int t = threadIdx.x;
        if (t < pairs) {
            const int left = t << (l + 1);
            part[left] = xor4(gh_mul_compact(part[left], fold_tabs + l * 512), part[left + (1 << l)]);
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
    uint32_t w[4] = {0, 0, 0, 0};
    for (int b = 0; b < n; ++b) {
        w[b >> 2] |= static_cast<uint32_t>(src[b]) << (8 * (b & 3));
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
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

}  // namespace dev
}  // namespace confkv
