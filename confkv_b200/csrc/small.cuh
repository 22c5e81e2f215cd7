// Small objects (at most kSmallMaxBlocks 16-byte blocks, or kWarpMaxBlocks
// when the batch plan routes mid objects here) in batched calls:
// one warp seals or opens a whole object, so a small object costs no
// block-wide fold, no barrier and no atomics, and many of them run side by
// side on every SM.
//
// Lane l takes blocks base + 32 r + l of row r (a warp row is 512
// contiguous bytes), base = n - 32 * rows <= 0 so the rows end at the
// object's end; lane chains q_l = sum_r C H^(32 (rows-1-r)) (the replicated
// H^32 table), then a 5-level shuffle fold gives sum_l q_l H^(31-l) =
// sum_i C_i H^(n-1-i), and GHASH = that * H^2 + L * H. Shared memory (the
// batched seal and open-CTR kernels switch to it after their chunks):
//   [0, 128K)          AES T-tables, replicated per lane
//   [128K, 192K)       H^32, replicated 4-bit table
//   [192K, 224K)       compact 4-bit tables of H^8, H^1, H^2, H^4
// H^16 (fold level 4) is read from the key's global tables.
#pragma once

#include "kernels.cuh"

namespace confkv {
namespace dev {

// Objects up to 16 KiB always. A warp's rows are serial, so a batch of fewer
// larger objects than warps ends on one warp's long chain (64 KiB objects ran
// at half the rate of 512-thread tiles).
constexpr uint64_t kSmallMaxBlocks = 1024;
// Objects of kSmallMaxBlocks + 1 .. kWarpMaxBlocks blocks ("mid" objects,
// up to 32 KiB) take the same warp path when the batch has enough of them
// (the batch plan decides, kMidAlphaSeal / kMidAlphaOpen); the warp code
// handles any length.
constexpr uint64_t kWarpMaxBlocks = 2048;
constexpr uint32_t kSmallGh = kAesBytes;
constexpr uint32_t kSmallFold = kAesBytes + kGhBytes;
constexpr uint32_t kSmallSmem = kSmallFold + 4 * 8192u;

// Compact table of fold level k (H^(2^k)) for the small-object fold.
__device__ __forceinline__ const uint4* small_fold_table(const uint8_t* smem, const uint4* pow2, int k)
{
    const uint4* ft = reinterpret_cast<const uint4*>(smem + kSmallFold);
    return k == 4 ? pow2 + 4 * 512 : (k == 3 ? ft : ft + (k + 1) * 512);
}

// Compact tables of H^8, H^1, H^2, H^4 into the fold slots. All threads.
__device__ __forceinline__ void fill_small_fold(uint8_t* smem, const uint4* pow2)
{
    uint4* ft = reinterpret_cast<uint4*>(smem + kSmallFold);
    fill_smem<512>(ft, pow2 + 3 * 512);       // slot 0: H^8
    fill_smem<3 * 512>(ft + 512, pow2);       // slots 1..3: H^1, H^2, H^4
}

// Fills all small-object tables above the AES region (open-CTR kernel).
__device__ __forceinline__ void small_fill_open_tables(uint8_t* smem, const uint4* pow2)
{
    fill_gh_smem(smem + kSmallGh, pow2 + 5 * 512);
    fill_small_fold(smem, pow2);
}

// GHASH of the object from the lane chains (returned in every lane):
// (sum_l q_l H^(31-l)) * H^2 + L * H. Only the lanes whose result is used
// multiply (16, 8, 4, 2, 1 at the fold levels, then lane 0), which keeps the
// shared-memory traffic of the fold at a fifth of an all-lane fold.
__device__ __forceinline__ uint4 small_ghash(uint4 q, uint64_t P, const uint8_t* smem, const uint4* pow2, int lane)
{
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const uint4 right = shfl_down4(q, 1 << k);
        if ((lane & ((2 << k) - 1)) == 0) {
            q = xor4(gh_mul_compact(q, small_fold_table(smem, pow2, k)), right);
        }
    }
    uint4 s = make_uint4(0, 0, 0, 0);
    if (lane == 0) {
        s = xor4(gh_mul_compact(q, small_fold_table(smem, pow2, 1)),
                 gh_mul_compact(be_to_raw(0ull, static_cast<unsigned long long>(P) * 8ull),
                                small_fold_table(smem, pow2, 0)));
    }
    return shfl4(s, 0);
}

// Geometry of an object split into warp rows.
struct SmallGeom {
    uint64_t P;
    int64_t n_full;
    int64_t rows;
    int64_t base;
};

__device__ __forceinline__ SmallGeom small_geom(uint64_t P)
{
    const int64_t n = static_cast<int64_t>(P / 16u + ((P & 15u) != 0));
    const int64_t rows = n == 0 ? 1 : (n + 31) / 32;
    return SmallGeom{P, static_cast<int64_t>(P / 16u), rows, n - 32 * rows};
}

// Seals one object with the calling warp (every lane calls it).
__device__ __forceinline__ void seal_object_warp(const BatchItem* it, const uint32_t* rk, const uint4* pow2,
                                                 const uint8_t* smem, int lane)
{
    const SmallGeom g = small_geom(it->plen);
    const uint8_t* src = it->src;
    uint8_t* frame = it->dst;
    uint8_t* ct = frame + 13;
    const uint32_t ivw[3] = {it->iv[0], it->iv[1], it->iv[2]};
    if (lane < 13) {
        frame[lane] = lane == 0 ? 1 : static_cast<uint8_t>(ivw[(lane - 1) >> 2] >> (8 * ((lane - 1) & 3)));
    }
    uint32_t lb[4];
    aes_lane_bases(lb, lane);
    const uint32_t lb_lo = static_cast<uint32_t>(lane & 7) << 4;
    const uint32_t lb_hi = 0x80u | lb_lo;
    const uint32_t s012[3] = {ivw[0] ^ rk[0], ivw[1] ^ rk[1], ivw[2] ^ rk[2]};
    const uint32_t so = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src) & 15u);
    const uint32_t sq = so >> 2;
    const uint32_t sfs = funnel_sel(so & 3u);
    const uint32_t co = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(ct) & 15u);
    const uint32_t cs = 16u - co;
    const uint32_t cq = (cs >> 2) & 3u;
    const uint32_t cfs = funnel_sel(cs & 3u);
    // check-free rows: every block full and inside; a misaligned source also
    // needs both aligned chunks of each block inside the object
    const int64_t lo = so == 0 ? 0 : 1;
    const int64_t hi = g.n_full - (so == 0 ? 0 : 1);
    uint4 q = make_uint4(0, 0, 0, 0);
    WarpCtrCache cc{0xffffffffu, 0u, {0u, 0u, 0u, 0u}};
#pragma unroll 1
    for (int64_t r = 0; r < g.rows; ++r) {
        const int64_t i0 = g.base + 32 * r;
        const int64_t i = i0 + lane;
        const uint32_t ctr = static_cast<uint32_t>(i) + 2u;
        uint32_t x[4];
        uint4 c;
        if (i0 >= lo && i0 + 32 <= hi) {
            const uint8_t* sp = src + static_cast<uint64_t>(i) * 16u;
            const uint4 p = so == 0 ? __ldg(reinterpret_cast<const uint4*>(sp))
                                    : window16(__ldg(reinterpret_cast<const uint4*>(sp - so)),
                                               __ldg(reinterpret_cast<const uint4*>(sp - so + 16)), sq, sfs);
            warp_ctr_keystream<0>(x, ctr, cc, s012, rk, lb);
            c = make_uint4(p.x ^ x[0], p.y ^ x[1], p.z ^ x[2], p.w ^ x[3]);
            if (co == 0) {
                *reinterpret_cast<uint4*>(ct + static_cast<uint64_t>(i) * 16u) = c;
            } else {
                store_funnel_rt(ct + static_cast<uint64_t>(i) * 16u, c, cs, cq, cfs, lane);
            }
        } else {
            const int nb = block_bytes(i, g.P);
            const uint4 p = load_pt_block<false>(src, i, g.P);
            warp_ctr_keystream<0>(x, ctr, cc, s012, rk, lb);
            c = mask_bytes(make_uint4(p.x ^ x[0], p.y ^ x[1], p.z ^ x[2], p.w ^ x[3]), nb);
            if (co == 0) {
                if (nb == 16) {
                    *reinterpret_cast<uint4*>(ct + static_cast<uint64_t>(i) * 16u) = c;
                } else if (nb > 0) {
                    store_bytes(ct + static_cast<uint64_t>(i) * 16u, c, 0, nb);
                }
            } else {
                store_ct_block_rt(ct, i, c, nb, g.P, cs, cq, cfs, lane);
            }
        }
        q = xor4(gh_mul_rep<kSmallGh>(q, lb_lo, lb_hi), c);
    }
    const uint4 s = small_ghash(q, g.P, smem, pow2, lane);
    uint32_t w[4] = {s012[0], s012[1], s012[2], bswap32(1u) ^ rk[3]};
    aes_rounds_smem<0>(w, rk, lb);
    const uint4 tag = xor4(s, make_uint4(w[0], w[1], w[2], w[3]));
    if (lane < 16) {
        ct[g.P + lane] = static_cast<uint8_t>(byte_of(tag, lane));
    }
}

// Opens one object with the calling warp: GHASH of the ciphertext, the tag
// and version check (written to *auth_ok), then CTR into the destination
// or, on failure, zeros. Every lane calls it.
__device__ __forceinline__ void open_object_warp(const BatchItem* it, const uint32_t* rk, const uint4* pow2,
                                                 const uint8_t* smem, int lane)
{
    const SmallGeom g = small_geom(it->plen);
    const uint8_t* frame = it->src;
    const uint64_t frame_len = it->capacity;
    uint8_t* dst = it->dst;
    const uint32_t lo_off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(frame + 13) & 15u);
    const uint32_t lq = lo_off >> 2;
    const uint32_t lfs = funnel_sel(lo_off & 3u);
    const uint32_t lb_lo = static_cast<uint32_t>(lane & 7) << 4;
    const uint32_t lb_hi = 0x80u | lb_lo;
    // check-free rows: blocks 1 .. n_full - 1, so both aligned chunks of each
    // block lie inside the frame (the tag follows the last block)
    auto ct_fast = [&](int64_t i) __attribute__((always_inline)) {
        const uint8_t* cp = frame + 13 + static_cast<uint64_t>(i) * 16u;
        return lo_off == 0 ? *reinterpret_cast<const uint4*>(cp)
                           : window16(*reinterpret_cast<const uint4*>(cp - lo_off),
                                      *reinterpret_cast<const uint4*>(cp - lo_off + 16), lq, lfs);
    };
    uint4 q = make_uint4(0, 0, 0, 0);
#pragma unroll 1
    for (int64_t r = 0; r < g.rows; ++r) {
        const int64_t i0 = g.base + 32 * r;
        const int64_t i = i0 + lane;
        const uint4 c = (i0 >= 1 && i0 + 32 <= g.n_full) ? ct_fast(i)
                                                          : ct_block_rt(frame, frame_len, i, g.P, lo_off, lq, lfs);
        q = xor4(gh_mul_rep<kSmallGh>(q, lb_lo, lb_hi), c);
    }
    const uint4 s = small_ghash(q, g.P, smem, pow2, lane);
    uint32_t lb[4];
    aes_lane_bases(lb, lane);
    const uint4 iv = load_bytes(frame + 1, 12);
    const uint32_t s012[3] = {iv.x ^ rk[0], iv.y ^ rk[1], iv.z ^ rk[2]};
    uint32_t w[4] = {s012[0], s012[1], s012[2], bswap32(1u) ^ rk[3]};
    aes_rounds_smem<0>(w, rk, lb);
    const uint4 expect = xor4(s, make_uint4(w[0], w[1], w[2], w[3]));
    // lane b < 16 compares tag byte b; OR over the lanes, constant time
    uint32_t diff = lane < 16 ? (byte_of(expect, lane) ^ static_cast<uint32_t>(frame[13 + g.P + lane])) : 0u;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        diff |= __shfl_xor_sync(0xffffffffu, diff, o);
    }
    const int ok = (frame[0] == 1) & (diff == 0);
    if (lane == 0) {
        *it->auth_ok = ok;
    }

    const uint32_t d_off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(dst) & 15u);
    const uint32_t ds = 16u - d_off;
    const uint32_t dq = (ds >> 2) & 3u;
    const uint32_t dfs = funnel_sel(ds & 3u);
    WarpCtrCache cc{0xffffffffu, 0u, {0u, 0u, 0u, 0u}};
#pragma unroll 1
    for (int64_t r = 0; r < g.rows; ++r) {
        const int64_t i0 = g.base + 32 * r;
        const int64_t i = i0 + lane;
        const int nb = block_bytes(i, g.P);
        uint8_t* dp = dst + static_cast<uint64_t>(i) * 16u;
        if (!ok) {
            if (nb == 16 && d_off == 0) {
                *reinterpret_cast<uint4*>(dp) = make_uint4(0, 0, 0, 0);
            } else if (nb > 0) {
                store_bytes(dp, make_uint4(0, 0, 0, 0), 0, nb);
            }
            continue;
        }
        uint32_t x[4];
        warp_ctr_keystream<0>(x, static_cast<uint32_t>(i) + 2u, cc, s012, rk, lb);
        if (i0 >= 1 && i0 + 32 <= g.n_full) {
            const uint4 c = ct_fast(i);
            const uint4 p = make_uint4(c.x ^ x[0], c.y ^ x[1], c.z ^ x[2], c.w ^ x[3]);
            if (d_off == 0) {
                *reinterpret_cast<uint4*>(dp) = p;
            } else {
                store_funnel_rt(dp, p, ds, dq, dfs, lane);
            }
        } else {
            const uint4 c = ct_block_rt(frame, frame_len, i, g.P, lo_off, lq, lfs);
            const uint4 p = make_uint4(c.x ^ x[0], c.y ^ x[1], c.z ^ x[2], c.w ^ x[3]);
            if (nb == 16 && d_off == 0) {
                *reinterpret_cast<uint4*>(dp) = p;
            } else if (nb > 0) {
                store_bytes(dp, p, 0, nb);
            }
        }
    }
}

}  // namespace dev
}  // namespace confkv
