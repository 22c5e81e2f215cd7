// Per-CTA tile bodies shared by the single-object kernels (one object, grid
// = its G tiles) and the batched kernels (many objects, persistent CTAs
// taking tiles from a queue).
//
// A tile of object P (n = ceil(P/16) blocks) is J rows of kHornerThreads
// blocks starting at block `base`: row r holds blocks base + r*T + t for
// thread t. Tiles are aligned to the END of the object -- tile c of G covers
// [n - (G-c) J T, n - (G-1-c) J T) -- so only tile 0 can start below block 0
// (those slots are skipped) and every tile's GHASH share is scaled by the same
// kind of power, H^((G-1-c) J T + 2).
#pragma once

#include "kernels.cuh"

namespace confkv {
namespace dev {

// ---------------------------------------------------------------- seal

struct SealTile {
    const uint8_t* src;  // plaintext
    uint8_t* ct;         // frame + 13
    uint64_t P;
    int64_t base;        // first block of row 0 (negative only in tile 0)
    int64_t rows;        // J
    uint32_t s012[3];    // IV words ^ rk[0..2]
    uint32_t store_r;    // byte part of the ciphertext store funnel (SQ < 4)
};

// Row warps of a seal tile: AES-CTR of the tile's blocks, ciphertext stores,
// and the thread's GHASH share Q_t = sum_r C_(r,t) H^(T (J-1-r)) (returned).
// Rows [r_a, r_a + 2 ngroups) hold only full blocks inside the object: they
// run the check-free two-row loop. The others (tile 0's leading padding, the
// row with the last partial block, leftovers) take generic_row. Rows are
// visited in order.
//
// SQ selects the ciphertext store: 4 = ciphertext pointer 16-B aligned;
// 0..3 = word part of the funnel that builds an aligned 16-B chunk from this
// lane's block and the next lane's (byte part in t.store_r). GH = false
// leaves out the GHASH chain (the batched seal's CTR pass; its GHASH pass
// reads the ciphertext back) and returns zero.
template <int SQ, bool PT_ALIGNED, bool GH = true>
__device__ __forceinline__ uint4 seal_rows(const SealTile& t, const uint32_t* rk, const uint4* pow2, int tid,
                                           int lane)
{
    constexpr int R = kSealChains;
    uint32_t lb[4];
    aes_lane_bases(lb, lane);
    const uint32_t lb_lo = static_cast<uint32_t>(lane & 7) << 4;
    const uint32_t lb_hi = 0x80u | lb_lo;
    const uint32_t rk3x = bswap32(rk[3]);
    const uint32_t fsel = funnel_sel(t.store_r);
    const uint32_t s = (SQ < 4) ? 4u * SQ + t.store_r : 16u;  // 16 - (ct & 15)
    const uint64_t P = t.P;
    const int64_t base = t.base;
    const int64_t rows = t.rows;
    constexpr int64_t T = kHornerThreads;
    constexpr uint64_t kRowBytes = static_cast<uint64_t>(T) * 16u;
    Chains<R> ch;
#pragma unroll
    for (int k = 0; k < R; ++k) {
        ch.q[k] = make_uint4(0, 0, 0, 0);
    }

    // The interior loop takes kPair = 2 rows per iteration; with R > 1 chains
    // it starts on an even row so row r lands in chain r mod R (R divides
    // kPair). A misaligned plaintext is read as the two aligned 16-byte
    // chunks around each block, so its interior blocks are 1 .. n_full - 2
    // (both chunks inside the object).
    constexpr int64_t kPair = 2;
    static_assert(kPair % R == 0, "chains must divide the rows per iteration");
    constexpr int64_t kLoBlock = PT_ALIGNED ? 0 : 1;
    const int64_t n_full = static_cast<int64_t>(P / 16u);
    const int64_t r_lo = base >= kLoBlock ? 0 : (kLoBlock - base + T - 1) / T;
    int64_t r_hi = (n_full - (PT_ALIGNED ? 0 : 1) - base) / T;
    r_hi = r_hi > rows ? rows : r_hi;
    const uint32_t src_off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(t.src) & 15u);
    const uint32_t src_q = src_off >> 2;
    const uint32_t src_fsel = funnel_sel(src_off & 3u);
    // With one chain (or none, GH = false) every row is in chain 0, so the
    // loop starts at r_lo whatever its parity.
    int64_t r_a = (R == 1 || !GH) ? r_lo : (r_lo + kPair - 1) / kPair * kPair;
    r_a = r_a > r_hi ? r_hi : r_a;
    const int64_t ngroups = r_hi > r_a ? (r_hi - r_a) / kPair : 0;

    auto generic_row = [&](int64_t r) __attribute__((always_inline)) {
        const int64_t i = base + r * T + tid;
        const int nb = block_bytes(i, P);
        const uint4 p = load_pt_block<PT_ALIGNED>(t.src, i, P);
        uint32_t x[4] = {t.s012[0], t.s012[1], t.s012[2], bswap32(static_cast<uint32_t>(i) + 2u) ^ rk[3]};
        aes_rounds_smem<kSealAes>(x, rk, lb);
        const uint4 c = mask_bytes(make_uint4(p.x ^ x[0], p.y ^ x[1], p.z ^ x[2], p.w ^ x[3]), nb);
        store_ct_block<SQ>(t.ct, i, c, nb, P, s, fsel, lane);
        if constexpr (GH) {
            chain_push_dyn<kSealGh, R>(ch, static_cast<int>(r % R), c, lb_lo, lb_hi);
        }
    };

    // Rows below r_pad hold no block of the object (tile 0's leading
    // padding): they would only push zeros into chains that are still zero.
    int64_t r = base < 0 ? (-base) / T : 0;
#pragma unroll 1
    for (; r < r_a; ++r) {
        generic_row(r);
    }
    if (ngroups > 0) {
        // Two rows per iteration: two AES chains (rounds 1-2 from the
        // counter cache), the GHASH chain, next pair's plaintext prefetched.
        const uint64_t i0 = static_cast<uint64_t>(base + r_a * T + tid);
        // aligned: the block itself; misaligned: the aligned chunk holding its first byte
        const uint8_t* sp = reinterpret_cast<const uint8_t*>(
            reinterpret_cast<uintptr_t>(t.src + i0 * 16u) & ~static_cast<uintptr_t>(PT_ALIGNED ? 0 : 15));
        uint8_t* cp = t.ct + i0 * 16u;
        uint32_t ctr = static_cast<uint32_t>(i0) + 2u;
        CtrCache cc{0xffffffffu, 0u, {0u, 0u, 0u, 0u}};
        auto ld = [](const uint8_t* q) __attribute__((always_inline)) {
            return __ldg(reinterpret_cast<const uint4*>(q));
        };
        uint4 pf0 = ld(sp);
        uint4 pf1 = ld(sp + kRowBytes);
        uint4 pg0 = PT_ALIGNED ? make_uint4(0, 0, 0, 0) : ld(sp + 16);
        uint4 pg1 = PT_ALIGNED ? make_uint4(0, 0, 0, 0) : ld(sp + kRowBytes + 16);
#pragma unroll 1
        for (int64_t g = 0; g < ngroups; ++g) {
            const uint4 p0 = PT_ALIGNED ? pf0 : window16(pf0, pg0, src_q, src_fsel);
            const uint4 p1 = PT_ALIGNED ? pf1 : window16(pf1, pg1, src_q, src_fsel);
            if (g + 1 < ngroups) {
                const uint8_t* nx = sp + 2 * kRowBytes;
                pf0 = ld(nx);
                pf1 = ld(nx + kRowBytes);
                if (!PT_ALIGNED) {
                    pg0 = ld(nx + 16);
                    pg1 = ld(nx + kRowBytes + 16);
                }
            }
            const uint4 m0 = GH ? gh_mul_rep<kSealGh>(ch.q[0], lb_lo, lb_hi) : make_uint4(0, 0, 0, 0);
            uint32_t x[4], y[4];
            aes_ctr2_cached<kSealAes>(x, y, ctr, ctr + static_cast<uint32_t>(T), cc, t.s012, rk3x, rk, lb);
            const uint4 c0 = make_uint4(p0.x ^ x[0], p0.y ^ x[1], p0.z ^ x[2], p0.w ^ x[3]);
            const uint4 c1 = make_uint4(p1.x ^ y[0], p1.y ^ y[1], p1.z ^ y[2], p1.w ^ y[3]);
            store_ct_interior<SQ>(cp, c0, s, fsel, lane);
            store_ct_interior<SQ>(cp + kRowBytes, c1, s, fsel, lane);
            if constexpr (!GH) {
                (void)m0;
            } else if constexpr (R == 1) {
                ch.q[0] = xor4(gh_mul_rep<kSealGh>(xor4(m0, c0), lb_lo, lb_hi), c1);
            } else {
                const uint4 m1 = gh_mul_rep<kSealGh>(ch.q[1], lb_lo, lb_hi);
                ch.q[0] = xor4(m0, c0);
                ch.q[1] = xor4(m1, c1);
            }
            sp += 2 * kRowBytes;
            cp += 2 * kRowBytes;
            ctr += 2u * static_cast<uint32_t>(T);
        }
        r = r_a + kPair * ngroups;
    }
#pragma unroll 1
    for (; r < rows; ++r) {
        generic_row(r);
    }
    if constexpr (R == 1) {
        return ch.q[0];
    } else {
        return chains_combine<R>(ch, rows, pow2 + kHornerLog2 * 512);
    }
}

// Power warp of a seal tile: E_K(J0) from the shared T-tables, L*H for the
// length block, and lane p's U_p = H^d x^(4p) with d = (G-1-c) J T + 2.
// ALU_POW: H^d on the integer pipes (warp_h_pow_alu), for the per-object
// kernels, whose tiles can be a single row.
template <bool ALU_POW = false>
__device__ __forceinline__ void seal_power(const uint32_t ivw[3], const uint32_t* rk, uint64_t P,
                                           unsigned long long d, const uint4* pow2, int lane, uint4& ej0,
                                           uint4& lh, unsigned long long& uhi, unsigned long long& ulo)
{
    uint32_t lb[4];
    aes_lane_bases(lb, lane);
    uint32_t w[4] = {ivw[0] ^ rk[0], ivw[1] ^ rk[1], ivw[2] ^ rk[2], bswap32(1u) ^ rk[3]};
    aes_rounds_smem<kSealAes>(w, rk, lb);
    ej0 = make_uint4(w[0], w[1], w[2], w[3]);
    lh = warp_gh_mul_global(be_to_raw(0ull, static_cast<unsigned long long>(P) * 8ull), pow2, lane);
    warp_lane_basis(ALU_POW ? warp_h_pow_alu(pow2, d, lane) : warp_h_pow(pow2, d, lane), lane, uhi, ulo);
}

// Shared-memory bytes of the fold tables that seal_fold stores over the
// AES region (levels kSealFoldSmemLevels .. kFoldLevels-1).
constexpr uint32_t kSealLateBytes = (kFoldLevels - kSealFoldSmemLevels) * 8192u;

// Fold of the kHornerThreads seal partials (all threads of the CTA call it,
// after a barrier that follows the part[] writes). Levels 0..2 use the tables
// staged in kSealFold; the tables of the later levels are loaded into
// registers now and stored over the AES region after levels 0..2, so their L2
// latency overlaps that work. The AES region's first kSealLateBytes are
// clobbered; part[0] holds the CTA's fold on return.
__device__ __forceinline__ void seal_fold(uint8_t* smem, uint4* part, const uint4* pow2, int tid)
{
    constexpr int kLate = (kFoldLevels - kSealFoldSmemLevels) * 512;
    constexpr int kPer = (kLate + kSealThreads - 1) / kSealThreads;
    uint4 late[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = tid + k * kSealThreads;
        late[k] = i < kLate ? __ldg(pow2 + kSealFoldSmemLevels * 512 + i) : make_uint4(0, 0, 0, 0);
    }
    fold_partials<kSealFoldSmemLevels>(part, reinterpret_cast<const uint4*>(smem + kSealFold), pow2, 0,
                                       kSealFoldSmemLevels);
    uint4* late_tabs = reinterpret_cast<uint4*>(smem + kSealAes);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        const int i = tid + k * kSealThreads;
        if (i < kLate) {
            late_tabs[i] = late[k];
        }
    }
    __syncthreads();
    fold_partials<kFoldLevels>(part, late_tabs, pow2, kSealFoldSmemLevels, kFoldLevels);
}

// ------------------------------------------------------- two-stage fold
//
// The persistent batched kernels fold a tile's kHornerThreads partials Q_t in
// two stages, so the row warps hand their tile over and start the next one
// without waiting for the tile's epilogue (the per-object open-GHASH kernel
// folds the same way, with one barrier):
//   row warps   warp w folds its 32 partials with levels 0..3 into
//               V_p = sum_{t in [16p, 16p+16)} Q_t H^(16p+15-t), p = 2w, 2w+1
//               (warp_fold_pairs);
//   power warp  folds V_0..V_31 with levels 4..8 into
//               sum_p V_p H^(16 (31-p)) = sum_t Q_t H^(511-t) (power_fold),
//               the value fold_partials leaves in part[0].

// Levels 0..3 of a warp's fold. At level k, lanes i < 16 >> k combine the
// values of lanes 2i and 2i+1 as v_2i H^(2^k) + v_(2i+1): the active lanes stay
// contiguous, so a lookup of the compact tables costs as few shared-memory
// wavefronts as in a full warp. Lanes 0 and 1 return V_2w and V_2w+1. The
// compact table of H^(2^k) is at ft + 512 slot(k), slot(k) = k, or
// (k + 1) & 3 when SMALL_SLOTS (the small-object order H^8, H^1, H^2, H^4).
template <bool SMALL_SLOTS>
__device__ __forceinline__ uint4 warp_fold_pairs(uint4 q, const uint4* ft, int lane)
{
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint4 a = shfl4(q, (2 * lane) & 31);
        const uint4 b = shfl4(q, (2 * lane + 1) & 31);
        if (lane < (16 >> k)) {
            q = xor4(gh_mul_compact(a, ft + 512 * (SMALL_SLOTS ? ((k + 1) & 3) : k)), b);
        }
    }
    return q;
}

// Levels 4..8 on the power warp: lane p holds V_p; t4 is the compact table of
// H^16, followed by those of H^32 .. H^256 (shared or global memory). Returns
// the tile's fold in every lane.
__device__ __forceinline__ uint4 power_fold(uint4 v, const uint4* t4, int lane)
{
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const uint4 right = shfl_down4(v, 1 << k);
        if ((lane & ((2 << k) - 1)) == 0) {
            v = xor4(gh_mul_compact(v, t4 + 512 * k), right);
        }
    }
    return shfl4(v, 0);
}

// ---------------------------------------------------------------- open

struct OpenTile {
    const uint8_t* frame;
    uint64_t frame_len;
    uint64_t P;
    int64_t base;
    int64_t rows;
    uint32_t load_r;     // byte part of the ciphertext load funnel
};

// Row warps of an open-GHASH tile: the thread's GHASH share over the
// ciphertext at frame + 13 with R chains (multiplier M = H^(R T)), combined
// with the compact H^T table `ht`. In the interior rows chains
// k < R - NALU multiply with the replicated table of M at shared offset GH
// (shared-memory pipe; 4-bit table, or the kGhW-bit window table when T5) and
// the others with clmul (integer pipes, M's operands `cm` read from the
// kernel parameters), keeping their value in clmul's integer domain until
// the interior rows end; S interior rows are read at a time, the next S
// prefetched. Edge rows use the table for every chain. Interior rows hold
// blocks 1 <= i < P/16, so both aligned chunks of every block lie inside the
// frame and no checks are needed.
template <int LQ, int R, int NALU, int S, bool T5 = false, uint32_t GH = kOpenGh>
__device__ __forceinline__ uint4 open_ghash_rows(const OpenTile& t, const uint4* ht, const ClmulConst* cm, int tid,
                                                 int lane)
{
    constexpr int kTabChains = R - NALU;
    const uint32_t lb_lo = static_cast<uint32_t>(lane & 7) << 4;
    const uint32_t lb_hi = 0x80u | lb_lo;
    const uint32_t fsel = funnel_sel(t.load_r);
    const uint64_t P = t.P;
    const int64_t base = t.base;
    const int64_t rows = t.rows;
    constexpr int64_t T = kHornerThreads;
    constexpr uint64_t kRowBytes = static_cast<uint64_t>(T) * 16u;
    Chains<R> ch;
#pragma unroll
    for (int k = 0; k < R; ++k) {
        ch.q[k] = make_uint4(0, 0, 0, 0);
    }

    const int64_t n_full = static_cast<int64_t>(P / 16u);
    const int64_t r_lo = base >= 1 ? 0 : (1 - base + T - 1) / T;
    int64_t r_hi = (n_full - base) / T;
    r_hi = r_hi > rows ? rows : r_hi;
    int64_t r_a = (r_lo + R - 1) / R * R;
    r_a = r_a > r_hi ? r_hi : r_a;
    const int64_t ngroups = r_hi > r_a ? (r_hi - r_a) / R : 0;

    auto generic_row = [&](int64_t r) __attribute__((always_inline)) {
        const int64_t i = base + r * T + tid;
        const uint4 c = ct_finish<LQ>(ct_prefetch<LQ>(t.frame, t.frame_len, i, P), t.frame, i, P, fsel);
        if constexpr (T5) {
            chain_push_dyn5<GH, R>(ch, static_cast<int>(r % R), c, lb_lo);
        } else {
            chain_push_dyn<GH, R>(ch, static_cast<int>(r % R), c, lb_lo, lb_hi);
        }
    };

    int64_t r = base < 0 ? (-base) / T : 0;  // rows below hold no block of the object
#pragma unroll 1
    for (; r < r_a; ++r) {
        generic_row(r);
    }
    if (ngroups > 0) {
        // Rows are read S at a time, the next step's rows prefetched into
        // registers during the current step's multiplies; a group of R rows
        // is R / S steps, unrolled so that every chain index is a
        // compile-time constant.
        static_assert(R % S == 0, "steps must tile a group of rows");
        const uint64_t i0 = static_cast<uint64_t>(base + r_a * T + tid);
        const uint8_t* cp = t.frame + 13 + i0 * 16u;
        if (LQ != 4) {
            cp = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(cp) & ~static_cast<uintptr_t>(15));
        }
        uint4 pd[S], pe[S];
#pragma unroll
        for (int k = 0; k < S; ++k) {
            pd[k] = *reinterpret_cast<const uint4*>(cp + k * kRowBytes);
            pe[k] = LQ != 4 ? *reinterpret_cast<const uint4*>(cp + k * kRowBytes + 16) : make_uint4(0, 0, 0, 0);
        }
        uint32_t xi[NALU > 0 ? NALU : 1][4];  // integer-domain values of the integer-pipe chains
#pragma unroll
        for (int k = kTabChains; k < R; ++k) {
            const uint32_t q[4] = {ch.q[k].x, ch.q[k].y, ch.q[k].z, ch.q[k].w};
            clmul_from_raw(q, xi[k - kTabChains]);
        }
#pragma unroll 1
        for (int64_t g = 0; g < ngroups; ++g) {
#pragma unroll
            for (int h = 0; h < R / S; ++h) {
                if constexpr (T5) {
                    // keeps the compiler from interleaving the steps' table
                    // multiplies (kGh5Groups loads each), which overflowed the registers
                    __syncwarp();
                }
                uint4 cd[S], ce[S];
#pragma unroll
                for (int k = 0; k < S; ++k) {
                    cd[k] = pd[k];
                    ce[k] = pe[k];
                }
                if (h + 1 < R / S || g + 1 < ngroups) {
                    const uint8_t* nx = cp + S * kRowBytes;
#pragma unroll
                    for (int k = 0; k < S; ++k) {
                        pd[k] = *reinterpret_cast<const uint4*>(nx + k * kRowBytes);
                        pe[k] = LQ != 4 ? *reinterpret_cast<const uint4*>(nx + k * kRowBytes + 16)
                                        : make_uint4(0, 0, 0, 0);
                    }
                }
#pragma unroll
                for (int k = 0; k < S; ++k) {
                    const int chain = h * S + k;
                    const CtRaw raw{cd[k], ce[k], true};
                    const uint4 c = ct_finish<LQ>(raw, t.frame, 0, P, fsel);
                    if (chain < kTabChains) {
                        if constexpr (T5) {
                            ch.q[chain] = xor4(gh_mul_rep5<GH>(ch.q[chain], lb_lo), c);
                        } else {
                            ch.q[chain] = xor4(gh_mul_rep<GH>(ch.q[chain], lb_lo, lb_hi), c);
                        }
                    } else {
                        const uint32_t craw[4] = {c.x, c.y, c.z, c.w};
                        uint32_t ci[4];
                        clmul_from_raw(craw, ci);
                        clmul_horner(xi[chain - kTabChains], *cm, ci);
                    }
                }
                cp += S * kRowBytes;
            }
        }
#pragma unroll
        for (int k = kTabChains; k < R; ++k) {
            uint32_t q[4];
            clmul_to_raw(xi[k - kTabChains], q);
            ch.q[k] = make_uint4(q[0], q[1], q[2], q[3]);
        }
        r = r_a + R * ngroups;
    }
#pragma unroll 1
    for (; r < rows; ++r) {
        generic_row(r);
    }
    return chains_combine<R>(ch, rows, ht);
}

// Power warp of an open-GHASH tile: E_K(J0) (IV read from the frame, cipher
// from the compact T-tables aes_t: global memory, or a shared copy when
// AES_SMEM), L*H and U_p = H^d x^(4p) (on the integer pipes when ALU_POW).
template <bool ALU_POW = false, bool AES_SMEM = false>
__device__ __forceinline__ void open_power(const uint8_t* frame, const uint32_t* aes_t, const uint32_t* rk,
                                           uint64_t P, unsigned long long d, const uint4* pow2, int lane,
                                           uint4& ej0, uint4& lh, unsigned long long& uhi, unsigned long long& ulo)
{
    const uint4 iv = load_bytes(frame + 1, 12);
    ej0 = aes_encrypt_compact<!AES_SMEM>(aes_t, rk, make_uint4(iv.x, iv.y, iv.z, bswap32(1u)));
    lh = warp_gh_mul_global(be_to_raw(0ull, static_cast<unsigned long long>(P) * 8ull), pow2, lane);
    warp_lane_basis(ALU_POW ? warp_h_pow_alu(pow2, d, lane) : warp_h_pow(pow2, d, lane), lane, uhi, ulo);
}

// Tag check of open: 1 when the version byte is 1 and the frame's tag equals
// S ^ L*H ^ E_K(J0) (all 16 bytes compared, differences OR-accumulated).
__device__ __forceinline__ int open_verdict(const uint8_t* frame, uint64_t P, unsigned long long shi,
                                            unsigned long long slo, uint4 lh, uint4 ej0)
{
    const uint4 expect = xor4(xor4(be_to_raw(shi, slo), lh), ej0);
    const uint8_t* tag = frame + 13 + P;
    uint32_t diff = 0;
    for (int b = 0; b < 16; ++b) {
        diff |= byte_of(expect, b) ^ static_cast<uint32_t>(tag[b]);
    }
    return (frame[0] == 1) & (diff == 0);
}

// ------------------------------------------------------------ open: CTR

struct CtrTile {
    const uint8_t* frame;
    uint64_t frame_len;
    uint8_t* dst;
    uint64_t P;
    int64_t base;        // block of row 0 (thread 0)
    int64_t rows;
    uint32_t s012[3];    // IV words ^ rk[0..2]
    uint32_t load_r;
};

// Zero dst's bytes of the tile's blocks (failed authentication).
template <bool PT_ALIGNED>
__device__ __forceinline__ void ctr_zero_rows(const CtrTile& t, int tid)
{
    for (int64_t r = t.base < 0 ? (-t.base) / kCtrThreads : 0; r < t.rows; ++r) {
        const int64_t i = t.base + r * kCtrThreads + tid;
        const int nb = block_bytes(i, t.P);
        uint8_t* d = t.dst + static_cast<uint64_t>(i) * 16u;
        if (PT_ALIGNED && nb == 16) {
            *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
        } else {
            for (int b = 0; b < nb; ++b) {
                d[b] = 0;
            }
        }
    }
}

// Decrypt a tile's rows (kCtrThreads blocks each) with the replicated AES
// tables at shared offset 0. Interior rows hold blocks 1 <= i < P/16 (block
// 0's aligned chunk may start before the frame) and run two rows per
// iteration with the next pair prefetched; the rest take generic_row.
template <int LQ, bool PT_ALIGNED>
__device__ __forceinline__ void ctr_rows(const CtrTile& t, const uint32_t* rk, int tid, int lane)
{
    constexpr int64_t T = kCtrThreads;
    constexpr uint64_t kRowBytes = static_cast<uint64_t>(T) * 16u;
    const uint64_t P = t.P;
    const int64_t base = t.base;
    const int64_t rows = t.rows;
    uint32_t lb[4];
    aes_lane_bases(lb, lane);
    const uint32_t rk3x = bswap32(rk[3]);
    const uint32_t fsel = funnel_sel(t.load_r);
    // misaligned destination: s = 16 - (dst & 15) for the funnel stores
    const uint32_t dst_s = 16u - static_cast<uint32_t>(reinterpret_cast<uintptr_t>(t.dst) & 15u);
    const uint32_t dst_q = (dst_s >> 2) & 3u;
    const uint32_t dst_fsel = funnel_sel(dst_s & 3u);

    auto store_pt = [&](int64_t i, uint4 p) __attribute__((always_inline)) {
        const int nb = block_bytes(i, P);
        uint8_t* d = t.dst + static_cast<uint64_t>(i) * 16u;
        if (PT_ALIGNED && nb == 16) {
            *reinterpret_cast<uint4*>(d) = p;
        } else if (nb > 0) {
            store_bytes(d, p, 0, nb);
        }
    };
    auto generic_row = [&](int64_t r) __attribute__((always_inline)) {
        const int64_t i = base + r * T + tid;
        const uint4 c = ct_finish<LQ>(ct_prefetch<LQ>(t.frame, t.frame_len, i, P), t.frame, i, P, fsel);
        uint32_t x[4] = {t.s012[0], t.s012[1], t.s012[2], bswap32(static_cast<uint32_t>(i) + 2u) ^ rk[3]};
        aes_rounds_smem<0>(x, rk, lb);
        store_pt(i, make_uint4(c.x ^ x[0], c.y ^ x[1], c.z ^ x[2], c.w ^ x[3]));
    };

    const int64_t n_full = static_cast<int64_t>(P / 16u);
    int64_t r_lo = base >= 1 ? 0 : (1 - base + T - 1) / T;
    int64_t r_hi = (n_full - base) / T;
    r_hi = r_hi > rows ? rows : r_hi;
    if (r_lo > r_hi) {
        r_lo = r_hi = rows;
    }
    int64_t r = base < 0 ? (-base) / T : 0;  // rows below hold no block of the object
#pragma unroll 1
    for (; r < r_lo; ++r) {
        generic_row(r);
    }
    const int64_t npair = (r_hi - r_lo) / 2;
    if (npair > 0) {
        const uint64_t i0 = static_cast<uint64_t>(base + r_lo * T + tid);
        const uint8_t* cp = t.frame + 13 + i0 * 16u;
        if (LQ != 4) {
            cp = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(cp) & ~static_cast<uintptr_t>(15));
        }
        uint8_t* dp = t.dst + i0 * 16u;
        uint32_t ctr = static_cast<uint32_t>(i0) + 2u;
        CtrCache cc{0xffffffffu, 0u, {0u, 0u, 0u, 0u}};
        uint4 pd0 = *reinterpret_cast<const uint4*>(cp);
        uint4 pe0 = LQ != 4 ? *reinterpret_cast<const uint4*>(cp + 16) : make_uint4(0, 0, 0, 0);
        uint4 pd1 = *reinterpret_cast<const uint4*>(cp + kRowBytes);
        uint4 pe1 = LQ != 4 ? *reinterpret_cast<const uint4*>(cp + kRowBytes + 16) : make_uint4(0, 0, 0, 0);
#pragma unroll 1
        for (int64_t k = 0; k < npair; ++k) {
            const CtRaw r0{pd0, pe0, true};
            const CtRaw r1{pd1, pe1, true};
            if (k + 1 < npair) {
                const uint8_t* nx = cp + 2 * kRowBytes;
                pd0 = *reinterpret_cast<const uint4*>(nx);
                pe0 = LQ != 4 ? *reinterpret_cast<const uint4*>(nx + 16) : make_uint4(0, 0, 0, 0);
                pd1 = *reinterpret_cast<const uint4*>(nx + kRowBytes);
                pe1 = LQ != 4 ? *reinterpret_cast<const uint4*>(nx + kRowBytes + 16) : make_uint4(0, 0, 0, 0);
            }
            uint32_t x[4], y[4];
            aes_ctr2_cached<0>(x, y, ctr, ctr + static_cast<uint32_t>(T), cc, t.s012, rk3x, rk, lb);
            const uint4 c0 = ct_finish<LQ>(r0, t.frame, 0, P, fsel);
            const uint4 c1 = ct_finish<LQ>(r1, t.frame, 0, P, fsel);
            const uint4 p0 = make_uint4(c0.x ^ x[0], c0.y ^ x[1], c0.z ^ x[2], c0.w ^ x[3]);
            const uint4 p1 = make_uint4(c1.x ^ y[0], c1.y ^ y[1], c1.z ^ y[2], c1.w ^ y[3]);
            if (PT_ALIGNED) {
                *reinterpret_cast<uint4*>(dp) = p0;
                *reinterpret_cast<uint4*>(dp + kRowBytes) = p1;
            } else {
                store_funnel_rt(dp, p0, dst_s, dst_q, dst_fsel, lane);
                store_funnel_rt(dp + kRowBytes, p1, dst_s, dst_q, dst_fsel, lane);
            }
            cp += 2 * kRowBytes;
            dp += 2 * kRowBytes;
            ctr += 2u * static_cast<uint32_t>(T);
        }
        r = r_lo + 2 * npair;
    }
#pragma unroll 1
    for (; r < rows; ++r) {
        generic_row(r);
    }
}

}  // namespace dev
}  // namespace confkv
