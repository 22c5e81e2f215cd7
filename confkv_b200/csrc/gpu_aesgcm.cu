// B200 (sm_100a) AES-128-GCM seal/open engine behind ConfKV's GPU C-ABI
// (experiments/gpu_kv_seal/gpu/gpu_aesgcm_api.h). Kernels live in
// kernels.cuh; this file holds the kernels' bodies, the key handle and the
// seven exported functions.
//
// Seal is ONE kernel per object (the reference enqueues about twenty: header,
// CTR, GHASH segments, sixteen combine launches and finalize,
// gpu_aesgcm.cu:1455-1623). Open is two kernels in stream order: GHASH + tag
// verification writes *auth_ok, then CTR decrypts or zero-fills
// (gpu_aesgcm.cu:1626-1776 semantics).
#include "gpu_aesgcm_api.h"

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "host_crypto.h"
#include "kernels.cuh"

namespace confkv {
namespace dev {

// ------------------------------------------------------------ seal kernel
//
// CTA c owns blocks [n - (G-c)*J*T, n - (G-1-c)*J*T) (only CTA 0 may start
// below block 0; those leading slots are skipped). In iteration it thread t
// handles block base + it*T + t, so a warp touches 512 contiguous bytes.
// Thread t's GHASH chain is Q_t = sum_it C * H^(T*(J-1-it)); the CTA's share
// of the tag hash is (sum_t Q_t H^(T-1-t)) * H^(d_c), d_c = n + 2 - e_c, where
// the power warp computes H^(d_c) while the other warps run the main loop.
//
// SQ selects the ciphertext store: 4 = ciphertext pointer 16-B aligned;
// 0..3 = word part of the funnel that builds an aligned 16-B chunk from this
// lane's block and the next lane's (byte part in a.store_r).
template <int SQ, bool PT_ALIGNED>
__global__ void __launch_bounds__(kSealThreads, 1) seal_kernel(const SealArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* aes_tab = smem + kSealAes;
    uint8_t* gh_tab = smem + kSealGh;
    uint4* part = reinterpret_cast<uint4*>(smem + kSealPart);
    uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kSealMisc);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    fill_aes_smem(aes_tab, a.kt.aes_t);
    fill_gh_smem(gh_tab, a.kt.gh_main);
    if (blockIdx.x == 0 && tid == 0) {
        a.frame[0] = 1;
        for (int b = 0; b < 12; ++b) {
            a.frame[1 + b] = static_cast<uint8_t>(a.ivw[b >> 2] >> (8 * (b & 3)));
        }
    }
    __syncthreads();

    const uint64_t P = a.plen;
    const int64_t n = a.nblocks;
    const int64_t span = static_cast<int64_t>(a.iters) * kHornerThreads;
    const int64_t base = n - static_cast<int64_t>(a.grid - blockIdx.x) * span;
    uint8_t* ct = a.frame + 13;

    unsigned long long uhi = 0, ulo = 0;  // power warp: U_p = M * x^(4p)
    uint4 q = make_uint4(0, 0, 0, 0);

    if (warp == kPowerWarp) {
        const unsigned long long d = static_cast<unsigned long long>(a.grid - 1 - blockIdx.x) *
                                         static_cast<unsigned long long>(span) + 2ull;
        const uint4 m = warp_h_pow(a.kt.gh_pow2, d, lane);
        warp_lane_basis(m, lane, uhi, ulo);
    } else {
        uint32_t lb[4];
        aes_lane_bases(lb, lane);
        const uint32_t lb_lo = static_cast<uint32_t>(lane & 7) << 4;
        const uint32_t lb_hi = 0x80u | lb_lo;
        const uint32_t w0 = a.ivw[0] ^ a.rk[0];
        const uint32_t w1 = a.ivw[1] ^ a.rk[1];
        const uint32_t w2 = a.ivw[2] ^ a.rk[2];
        const uint32_t fsel = funnel_sel(a.store_r);
        const uint32_t s = (SQ < 4) ? 4u * SQ + a.store_r : 16u;  // 16 - (ct & 15)

#pragma unroll 1
        for (uint32_t it = 0; it < a.iters; ++it) {
            const int64_t i = base + static_cast<int64_t>(it) * kHornerThreads + tid;
            const bool valid = i >= 0;
            const uint64_t off = static_cast<uint64_t>(i) * 16u;
            uint4 c = make_uint4(0, 0, 0, 0);
            int nbytes = 0;
            if (valid) {
                const uint64_t rem = P - off;
                nbytes = rem >= 16 ? 16 : static_cast<int>(rem);
                uint4 p;
                if (PT_ALIGNED && nbytes == 16) {
                    p = __ldg(reinterpret_cast<const uint4*>(a.src + off));
                } else {
                    p = load_bytes(a.src + off, nbytes);
                }
                uint32_t w[4] = {w0, w1, w2, bswap32(static_cast<uint32_t>(i) + 2u) ^ a.rk[3]};
                aes_rounds_smem(w, a.rk, aes_tab, lb);
                c = mask_bytes(make_uint4(p.x ^ w[0], p.y ^ w[1], p.z ^ w[2], p.w ^ w[3]), nbytes);
            }

            if (SQ == 4) {
                if (valid) {
                    if (nbytes == 16) {
                        *reinterpret_cast<uint4*>(ct + off) = c;
                    } else {
                        store_bytes(ct + off, c, 0, nbytes);
                    }
                }
            } else {
                // next lane's block words 0..SQ
                uint32_t nb[4];
#pragma unroll
                for (int k = 0; k <= SQ; ++k) {
                    nb[k] = __shfl_down_sync(0xffffffffu, word_of(c, k), 1);
                }
                const bool full = valid && lane < 31 && off + s + 16 <= P;
                const bool prev_full = valid && lane > 0 && i >= 1 && off + s <= P;
                if (full) {
                    const uint32_t sw[8] = {c.x, c.y, c.z, c.w, nb[0], SQ >= 1 ? nb[1] : 0u,
                                            SQ >= 2 ? nb[2] : 0u, SQ >= 3 ? nb[3] : 0u};
                    uint4 o;
                    o.x = funnel(sw[SQ + 0], sw[SQ + 1], fsel);
                    o.y = funnel(sw[SQ + 1], sw[SQ + 2], fsel);
                    o.z = funnel(sw[SQ + 2], sw[SQ + 3], fsel);
                    o.w = funnel(sw[SQ + 3], sw[SQ + 4], fsel);
                    *reinterpret_cast<uint4*>(ct + off + s) = o;
                } else if (valid) {
                    store_bytes(ct + off, c, static_cast<int>(s), nbytes);
                }
                if (valid && !prev_full) {
                    store_bytes(ct + off, c, 0, nbytes < static_cast<int>(s) ? nbytes : static_cast<int>(s));
                }
            }

            if (valid) {
                q = xor4(gh_mul_rep(q, gh_tab, lb_lo, lb_hi), c);
            }
        }
        part[tid] = q;
    }
    __syncthreads();

    // Stage the fold tables H^(2^l), l < kFoldLevels, over the GHASH region.
    uint4* fold_tabs = reinterpret_cast<uint4*>(gh_tab);
    for (int i = tid; i < kFoldLevels * 512; i += blockDim.x) {
        fold_tabs[i] = __ldg(a.kt.gh_pow2 + i);
    }
    __syncthreads();
    fold_partials(part, fold_tabs);

    if (warp == kPowerWarp) {
        unsigned long long rhi, rlo;
        warp_generic_mul(part[0], uhi, ulo, lane, rhi, rlo);
        unsigned int ticket = 0;
        if (lane == 0) {
            atomicXor(&a.slot->acc_hi, rhi);
            atomicXor(&a.slot->acc_lo, rlo);
            __threadfence();
            ticket = atomicAdd(&a.slot->ticket, 1u);
        }
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == a.grid - 1) {
            __threadfence();
            unsigned long long shi = 0, slo = 0;
            if (lane == 0) {
                shi = atomicXor(&a.slot->acc_hi, 0ull);
                slo = atomicXor(&a.slot->acc_lo, 0ull);
            }
            shi = __shfl_sync(0xffffffffu, shi, 0);
            slo = __shfl_sync(0xffffffffu, slo, 0);
            // length block [0^64 || 8P] times H
            const uint4 lenblk = be_to_raw(0ull, static_cast<unsigned long long>(P) * 8ull);
            const uint4 lh = warp_gh_mul_global(lenblk, a.kt.gh_pow2, lane);
            uint32_t lb[4];
            aes_lane_bases(lb, lane);
            uint32_t w[4] = {a.ivw[0] ^ a.rk[0], a.ivw[1] ^ a.rk[1], a.ivw[2] ^ a.rk[2],
                             bswap32(1u) ^ a.rk[3]};
            aes_rounds_smem(w, a.rk, aes_tab, lb);
            const uint4 tag = xor4(xor4(be_to_raw(shi, slo), lh), make_uint4(w[0], w[1], w[2], w[3]));
            if (lane < 16) {
                ct[P + lane] = static_cast<uint8_t>(byte_of(tag, lane));
            }
            if (lane == 0) {
                a.slot->acc_hi = 0;
                a.slot->acc_lo = 0;
                a.slot->ticket = 0;
            }
        }
    }
    (void)misc;
}

// Zero-length seal: header + tag = E_K(J0) (GHASH of nothing is 0).
__global__ void seal_empty_kernel(const SealArgs a)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) {
        return;
    }
    a.frame[0] = 1;
    for (int b = 0; b < 12; ++b) {
        a.frame[1 + b] = static_cast<uint8_t>(a.ivw[b >> 2] >> (8 * (b & 3)));
    }
    const uint4 e = aes_encrypt_gmem(a.kt.aes_t, a.rk, make_uint4(a.ivw[0], a.ivw[1], a.ivw[2], bswap32(1u)));
    for (int b = 0; b < 16; ++b) {
        a.frame[13 + b] = static_cast<uint8_t>(byte_of(e, b));
    }
}

// ---------------------------------------------------- open: GHASH + verify
//
// Same CTA/thread partition and fold as seal_kernel, over the ciphertext at
// frame + 13. LQ = word part of the load funnel (byte part a.load_r), 4 when
// the ciphertext is 16-B aligned. Each lane reads the two aligned 16-B chunks
// covering its block when both lie inside the frame buffer, else bytes.
template <int LQ>
__device__ __forceinline__ uint4 load_ct_block(const uint8_t* frame, uint64_t frame_len,
                                               uint64_t off, int nbytes, uint32_t fsel)
{
    const uint8_t* ct = frame + 13;
    if (nbytes == 16) {
        if (LQ == 4) {
            return *reinterpret_cast<const uint4*>(ct + off);
        }
        const uint64_t lag = 4u * LQ + 0u;  // word part; byte part folded into fsel
        (void)lag;
        const uint8_t* c0 = reinterpret_cast<const uint8_t*>(
            reinterpret_cast<uintptr_t>(ct + off) & ~static_cast<uintptr_t>(15));
        if (c0 >= frame && c0 + 32 <= frame + frame_len) {
            const uint4 d = *reinterpret_cast<const uint4*>(c0);
            const uint4 e = *reinterpret_cast<const uint4*>(c0 + 16);
            const uint32_t sw[8] = {d.x, d.y, d.z, d.w, e.x, e.y, e.z, e.w};
            return make_uint4(funnel(sw[LQ], sw[LQ + 1], fsel), funnel(sw[LQ + 1], sw[LQ + 2], fsel),
                              funnel(sw[LQ + 2], sw[LQ + 3], fsel), funnel(sw[LQ + 3], sw[LQ + 4], fsel));
        }
    }
    return load_bytes(ct + off, nbytes);
}

template <int LQ>
__global__ void __launch_bounds__(kSealThreads, 1) open_ghash_kernel(const OpenArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* gh_tab = smem + kOpenGh;
    uint4* part = reinterpret_cast<uint4*>(smem + kOpenPart);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    fill_gh_smem(gh_tab, a.kt.gh_main);
    __syncthreads();

    const uint64_t P = a.plen;
    const int64_t n = a.nblocks;
    const int64_t span = static_cast<int64_t>(a.iters) * kHornerThreads;
    const int64_t base = n - static_cast<int64_t>(a.grid - blockIdx.x) * span;

    unsigned long long uhi = 0, ulo = 0;
    uint4 q = make_uint4(0, 0, 0, 0);

    if (warp == kPowerWarp) {
        const unsigned long long d = static_cast<unsigned long long>(a.grid - 1 - blockIdx.x) *
                                         static_cast<unsigned long long>(span) + 2ull;
        const uint4 m = warp_h_pow(a.kt.gh_pow2, d, lane);
        warp_lane_basis(m, lane, uhi, ulo);
    } else {
        const uint32_t lb_lo = static_cast<uint32_t>(lane & 7) << 4;
        const uint32_t lb_hi = 0x80u | lb_lo;
        const uint32_t fsel = funnel_sel(a.load_r);
#pragma unroll 1
        for (uint32_t it = 0; it < a.iters; ++it) {
            const int64_t i = base + static_cast<int64_t>(it) * kHornerThreads + tid;
            if (i >= 0) {
                const uint64_t off = static_cast<uint64_t>(i) * 16u;
                const uint64_t rem = P - off;
                const int nbytes = rem >= 16 ? 16 : static_cast<int>(rem);
                const uint4 c = load_ct_block<LQ>(a.frame, a.frame_len, off, nbytes, fsel);
                q = xor4(gh_mul_rep(q, gh_tab, lb_lo, lb_hi), c);
            }
        }
        part[tid] = q;
    }
    __syncthreads();

    uint4* fold_tabs = reinterpret_cast<uint4*>(gh_tab);
    for (int i = tid; i < kFoldLevels * 512; i += blockDim.x) {
        fold_tabs[i] = __ldg(a.kt.gh_pow2 + i);
    }
    __syncthreads();
    fold_partials(part, fold_tabs);

    if (warp == kPowerWarp) {
        unsigned long long rhi, rlo;
        warp_generic_mul(part[0], uhi, ulo, lane, rhi, rlo);
        unsigned int ticket = 0;
        if (lane == 0) {
            atomicXor(&a.slot->acc_hi, rhi);
            atomicXor(&a.slot->acc_lo, rlo);
            __threadfence();
            ticket = atomicAdd(&a.slot->ticket, 1u);
        }
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == a.grid - 1) {
            __threadfence();
            unsigned long long shi = 0, slo = 0;
            if (lane == 0) {
                shi = atomicXor(&a.slot->acc_hi, 0ull);
                slo = atomicXor(&a.slot->acc_lo, 0ull);
            }
            shi = __shfl_sync(0xffffffffu, shi, 0);
            slo = __shfl_sync(0xffffffffu, slo, 0);
            const uint4 lenblk = be_to_raw(0ull, static_cast<unsigned long long>(P) * 8ull);
            const uint4 lh = warp_gh_mul_global(lenblk, a.kt.gh_pow2, lane);
            if (lane == 0) {
                const uint4 iv = load_bytes(a.frame + 1, 12);
                const uint4 e = aes_encrypt_gmem(a.kt.aes_t, a.rk, make_uint4(iv.x, iv.y, iv.z, bswap32(1u)));
                const uint4 expect = xor4(xor4(be_to_raw(shi, slo), lh), e);
                const uint8_t* tag = a.frame + 13 + P;
                uint32_t diff = 0;
                for (int b = 0; b < 16; ++b) {
                    diff |= byte_of(expect, b) ^ static_cast<uint32_t>(tag[b]);
                }
                const int ok = (a.frame[0] == 1) & (diff == 0);
                *a.auth_ok = ok;
                a.slot->acc_hi = 0;
                a.slot->acc_lo = 0;
                a.slot->ticket = 0;
            }
        }
    }
}

// Zero-length open: only the version byte and tag = E_K(J0) to check.
__global__ void open_empty_kernel(const OpenArgs a)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) {
        return;
    }
    const uint4 iv = load_bytes(a.frame + 1, 12);
    const uint4 e = aes_encrypt_gmem(a.kt.aes_t, a.rk, make_uint4(iv.x, iv.y, iv.z, bswap32(1u)));
    uint32_t diff = 0;
    for (int b = 0; b < 16; ++b) {
        diff |= byte_of(e, b) ^ static_cast<uint32_t>(a.frame[13 + b]);
    }
    *a.auth_ok = (a.frame[0] == 1) & (diff == 0);
}

// ------------------------------------------------------ open: gated CTR
//
// Reads *auth_ok (written by open_ghash_kernel earlier on the same stream).
// Authentic: plaintext = ciphertext ^ keystream. Otherwise dst[0, P) is
// zero-filled and no keystream is produced.
template <int LQ, bool PT_ALIGNED>
__global__ void __launch_bounds__(kCtrThreads, 1) open_ctr_kernel(const CtrArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const uint64_t P = a.plen;
    const uint64_t n = a.nblocks;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    const int ok = *reinterpret_cast<const volatile int*>(a.auth_ok);

    if (!ok) {
        for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
            const uint64_t off = i * 16u;
            const uint64_t rem = P - off;
            const int nbytes = rem >= 16 ? 16 : static_cast<int>(rem);
            if (PT_ALIGNED && nbytes == 16) {
                *reinterpret_cast<uint4*>(a.dst + off) = make_uint4(0, 0, 0, 0);
            } else {
                for (int b = 0; b < nbytes; ++b) {
                    a.dst[off + b] = 0;
                }
            }
        }
        return;
    }

    uint8_t* aes_tab = smem;
    fill_aes_smem(aes_tab, a.aes_t);
    __syncthreads();

    const int lane = threadIdx.x & 31;
    uint32_t lb[4];
    aes_lane_bases(lb, lane);
    const uint4 iv = load_bytes(a.frame + 1, 12);
    const uint32_t w0 = iv.x ^ a.rk[0];
    const uint32_t w1 = iv.y ^ a.rk[1];
    const uint32_t w2 = iv.z ^ a.rk[2];
    const uint32_t fsel = funnel_sel(a.load_r);

#pragma unroll 1
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t off = i * 16u;
        const uint64_t rem = P - off;
        const int nbytes = rem >= 16 ? 16 : static_cast<int>(rem);
        const uint4 c = load_ct_block<LQ>(a.frame, a.frame_len, off, nbytes, fsel);
        uint32_t w[4] = {w0, w1, w2, bswap32(static_cast<uint32_t>(i) + 2u) ^ a.rk[3]};
        aes_rounds_smem(w, a.rk, aes_tab, lb);
        const uint4 p = make_uint4(c.x ^ w[0], c.y ^ w[1], c.z ^ w[2], c.w ^ w[3]);
        if (PT_ALIGNED && nbytes == 16) {
            *reinterpret_cast<uint4*>(a.dst + off) = p;
        } else {
            store_bytes(a.dst + off, p, 0, nbytes);
        }
    }
}

}  // namespace dev
}  // namespace confkv

// ====================================================================== host

namespace {

using confkv::Gf128;
namespace dev = confkv::dev;

constexpr size_t kFrameOverhead = 29;
constexpr uint64_t kMaxBlocks = 0xfffffffeull;
constexpr int kSlots = 64;
constexpr int kMaxDevices = 64;

struct KeyHandle {
    int device = 0;
    int num_sms = 0;
    uint32_t rk[confkv::kRoundKeyWords];
    uint8_t* d_mem = nullptr;  // one allocation: tables + slots
    dev::KeyTables kt{};
    dev::Slot* slots = nullptr;
    std::atomic<uint32_t> next_slot{0};
};

class DeviceGuard {
public:
    explicit DeviceGuard(int target)
    {
        if (cudaGetDevice(&old_) != cudaSuccess) {
            ok_ = false;
            return;
        }
        if (old_ != target) {
            ok_ = cudaSetDevice(target) == cudaSuccess;
            changed_ = ok_;
        }
    }
    ~DeviceGuard()
    {
        if (changed_) {
            cudaSetDevice(old_);
        }
    }
    bool ok() const { return ok_; }

private:
    int old_ = 0;
    bool changed_ = false;
    bool ok_ = true;
};

int cuda_rc(cudaError_t e)
{
    return e == cudaSuccess ? LMCACHE_GPU_AESGCM_OK : LMCACHE_GPU_AESGCM_ERR_CUDA;
}

// Host-side fault injection for tests: CONFKV_B200_FAIL_ALLOC=1 makes
// key_create report an allocation failure before touching the device.
bool alloc_fault_injected()
{
    const char* v = std::getenv("CONFKV_B200_FAIL_ALLOC");
    return v != nullptr && v[0] == '1';
}

template <class K>
cudaError_t allow_smem(K kernel, uint32_t bytes)
{
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bytes));
}

// Opt every kernel instantiation into its dynamic shared memory once per device.
cudaError_t configure_device(int device)
{
    static std::once_flag flags[kMaxDevices];
    static cudaError_t results[kMaxDevices];
    if (device < 0 || device >= kMaxDevices) {
        return cudaErrorInvalidDevice;
    }
    std::call_once(flags[device], [device]() {
        cudaError_t e = cudaSuccess;
        auto chk = [&e](cudaError_t r) {
            if (e == cudaSuccess) {
                e = r;
            }
        };
        chk(allow_smem(dev::seal_kernel<0, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<1, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<2, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<3, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<4, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<0, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<1, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<2, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<3, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_kernel<4, false>, dev::kSealSmem));
        chk(allow_smem(dev::open_ghash_kernel<0>, dev::kOpenSmem));
        chk(allow_smem(dev::open_ghash_kernel<1>, dev::kOpenSmem));
        chk(allow_smem(dev::open_ghash_kernel<2>, dev::kOpenSmem));
        chk(allow_smem(dev::open_ghash_kernel<3>, dev::kOpenSmem));
        chk(allow_smem(dev::open_ghash_kernel<4>, dev::kOpenSmem));
        chk(allow_smem(dev::open_ctr_kernel<0, true>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<1, true>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<2, true>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<3, true>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<4, true>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<0, false>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<1, false>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<2, false>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<3, false>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ctr_kernel<4, false>, dev::kCtrSmem));
        results[device] = e;
    });
    return results[device];
}

uint32_t le_word(const uint8_t* p)
{
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
           (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
}

// Seal/open-GHASH grid: J iterations of kHornerThreads blocks per CTA, at
// most one CTA per SM, G = ceil(n / (J*T)).
void horner_grid(uint64_t n, int num_sms, uint32_t& iters, uint32_t& grid)
{
    const uint64_t per_wave = static_cast<uint64_t>(num_sms) * dev::kHornerThreads;
    uint64_t j = (n + per_wave - 1) / per_wave;
    if (j == 0) {
        j = 1;
    }
    const uint64_t span = j * dev::kHornerThreads;
    iters = static_cast<uint32_t>(j);
    grid = static_cast<uint32_t>((n + span - 1) / span);
}

dev::Slot* take_slot(KeyHandle* h)
{
    return h->slots + (h->next_slot.fetch_add(1, std::memory_order_relaxed) % kSlots);
}

template <int SQ, bool A>
cudaError_t launch_seal_t(const dev::SealArgs& args, cudaStream_t s)
{
    dev::seal_kernel<SQ, A><<<args.grid, dev::kSealThreads, dev::kSealSmem, s>>>(args);
    return cudaGetLastError();
}

template <int LQ>
cudaError_t launch_open_ghash_t(const dev::OpenArgs& args, cudaStream_t s)
{
    dev::open_ghash_kernel<LQ><<<args.grid, dev::kSealThreads, dev::kOpenSmem, s>>>(args);
    return cudaGetLastError();
}

template <int LQ, bool A>
cudaError_t launch_open_ctr_t(const dev::CtrArgs& args, uint32_t grid, cudaStream_t s)
{
    dev::open_ctr_kernel<LQ, A><<<grid, dev::kCtrThreads, dev::kCtrSmem, s>>>(args);
    return cudaGetLastError();
}

}  // namespace

extern "C" size_t lmcache_gpu_aesgcm_frame_size(size_t plaintext_len)
{
    return plaintext_len + kFrameOverhead;
}

extern "C" int lmcache_gpu_aes128gcm_key_create(const uint8_t* key, size_t key_len, int device,
                                                lmcache_gpu_aesgcm_key_t* out)
{
    if (key == nullptr || out == nullptr || key_len != 16) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    if (alloc_fault_injected()) {
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }
    DeviceGuard guard(device);
    if (!guard.ok()) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    if (configure_device(device) != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }

    auto* h = new (std::nothrow) KeyHandle();
    if (h == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }
    h->device = device;
    if (cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        h->num_sms <= 0) {
        delete h;
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }

    // Host precomputation: round keys, H = E_K(0^128), T-tables, GHASH tables.
    confkv::aes128_expand_le(key, h->rk);
    uint8_t zero[16] = {0};
    uint8_t hbytes[16];
    confkv::aes128_encrypt_block(h->rk, zero, hbytes);
    const Gf128 H = confkv::gf_load(hbytes);

    constexpr size_t kAesT = 4 * 256 * sizeof(uint32_t);
    constexpr size_t kTab = confkv::kGhashTableBytes;
    const size_t off_main = kAesT;
    const size_t off_pow2 = off_main + kTab;
    const size_t off_slots = off_pow2 + kTab * confkv::kPow2Tables;
    const size_t total = off_slots + sizeof(dev::Slot) * kSlots;

    uint8_t* host = new (std::nothrow) uint8_t[total];
    if (host == nullptr) {
        delete h;
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }
    std::memset(host, 0, total);
    confkv::aes_t_tables(reinterpret_cast<uint32_t(*)[256]>(host));
    confkv::ghash_table(confkv::gf_pow(H, dev::kHornerThreads), host + off_main);
    Gf128 p = H;
    for (int k = 0; k < confkv::kPow2Tables; ++k) {
        confkv::ghash_table(p, host + off_pow2 + kTab * k);
        p = confkv::gf_mul(p, p);
    }

    if (cudaMalloc(&h->d_mem, total) != cudaSuccess) {
        delete[] host;
        delete h;
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }
    const cudaError_t e = cudaMemcpy(h->d_mem, host, total, cudaMemcpyHostToDevice);
    delete[] host;
    if (e != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(h->d_mem);
        delete h;
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    h->kt.aes_t = reinterpret_cast<const uint32_t*>(h->d_mem);
    h->kt.gh_main = reinterpret_cast<const uint4*>(h->d_mem + off_main);
    h->kt.gh_pow2 = reinterpret_cast<const uint4*>(h->d_mem + off_pow2);
    h->slots = reinterpret_cast<dev::Slot*>(h->d_mem + off_slots);
    *out = reinterpret_cast<lmcache_gpu_aesgcm_key_t>(h);
    return LMCACHE_GPU_AESGCM_OK;
}

extern "C" int lmcache_gpu_aes128gcm_key_destroy(lmcache_gpu_aesgcm_key_t key)
{
    if (key == nullptr) {
        return LMCACHE_GPU_AESGCM_OK;
    }
    auto* h = reinterpret_cast<KeyHandle*>(key);
    {
        DeviceGuard guard(h->device);
        if (h->d_mem != nullptr) {
            cudaFree(h->d_mem);
        }
    }
    std::memset(h->rk, 0, sizeof(h->rk));
    delete h;
    return LMCACHE_GPU_AESGCM_OK;
}

extern "C" int lmcache_gpu_aes128gcm_reserve(lmcache_gpu_aesgcm_key_t key, size_t max_plaintext_len)
{
    (void)max_plaintext_len;
    if (key == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    return LMCACHE_GPU_AESGCM_OK;
}

extern "C" int lmcache_gpu_aes128gcm_seal_async(lmcache_gpu_aesgcm_key_t key, const void* src,
                                                size_t plaintext_len, void* dst, size_t dst_capacity,
                                                const uint8_t* iv, void* stream_ptr)
{
    if (key == nullptr || src == nullptr || dst == nullptr || iv == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    if (plaintext_len > SIZE_MAX - kFrameOverhead ||
        dst_capacity < lmcache_gpu_aesgcm_frame_size(plaintext_len)) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    const uint64_t n = (static_cast<uint64_t>(plaintext_len) + 15u) / 16u;
    if (n > kMaxBlocks) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    auto* h = reinterpret_cast<KeyHandle*>(key);
    DeviceGuard guard(h->device);
    if (!guard.ok()) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_ptr);

    dev::SealArgs args{};
    args.src = static_cast<const uint8_t*>(src);
    args.frame = static_cast<uint8_t*>(dst);
    args.plen = plaintext_len;
    args.nblocks = static_cast<uint32_t>(n);
    for (int k = 0; k < 3; ++k) {
        args.ivw[k] = le_word(iv + 4 * k);
    }
    std::memcpy(args.rk, h->rk, sizeof(args.rk));
    args.kt = h->kt;

    if (n == 0) {
        args.grid = 1;
        dev::seal_empty_kernel<<<1, 32, 0, s>>>(args);
        return cuda_rc(cudaGetLastError());
    }
    horner_grid(n, h->num_sms, args.iters, args.grid);
    args.slot = take_slot(h);

    const uintptr_t ct = reinterpret_cast<uintptr_t>(dst) + 13u;
    const uint32_t off = static_cast<uint32_t>(ct & 15u);
    const bool pt_aligned = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    int sq = 4;
    if (off != 0) {
        const uint32_t sh = 16u - off;
        sq = static_cast<int>(sh >> 2);
        args.store_r = sh & 3u;
    }
    cudaError_t e;
    if (pt_aligned) {
        switch (sq) {
        case 0: e = launch_seal_t<0, true>(args, s); break;
        case 1: e = launch_seal_t<1, true>(args, s); break;
        case 2: e = launch_seal_t<2, true>(args, s); break;
        case 3: e = launch_seal_t<3, true>(args, s); break;
        default: e = launch_seal_t<4, true>(args, s); break;
        }
    } else {
        switch (sq) {
        case 0: e = launch_seal_t<0, false>(args, s); break;
        case 1: e = launch_seal_t<1, false>(args, s); break;
        case 2: e = launch_seal_t<2, false>(args, s); break;
        case 3: e = launch_seal_t<3, false>(args, s); break;
        default: e = launch_seal_t<4, false>(args, s); break;
        }
    }
    return cuda_rc(e);
}

extern "C" int lmcache_gpu_aes128gcm_open_async(lmcache_gpu_aesgcm_key_t key, const void* src,
                                                size_t frame_len, void* dst, size_t plaintext_len,
                                                int* auth_ok, void* stream_ptr)
{
    if (key == nullptr || src == nullptr || dst == nullptr || auth_ok == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    if (plaintext_len > SIZE_MAX - kFrameOverhead ||
        frame_len < lmcache_gpu_aesgcm_frame_size(plaintext_len)) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    const uint64_t n = (static_cast<uint64_t>(plaintext_len) + 15u) / 16u;
    if (n > kMaxBlocks) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    auto* h = reinterpret_cast<KeyHandle*>(key);
    DeviceGuard guard(h->device);
    if (!guard.ok()) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_ptr);

    dev::OpenArgs oa{};
    oa.frame = static_cast<const uint8_t*>(src);
    oa.frame_len = frame_len;
    oa.plen = plaintext_len;
    oa.nblocks = static_cast<uint32_t>(n);
    std::memcpy(oa.rk, h->rk, sizeof(oa.rk));
    oa.kt = h->kt;
    oa.auth_ok = auth_ok;

    if (n == 0) {
        dev::open_empty_kernel<<<1, 32, 0, s>>>(oa);
        return cuda_rc(cudaGetLastError());
    }
    horner_grid(n, h->num_sms, oa.iters, oa.grid);
    oa.slot = take_slot(h);

    const uintptr_t ct = reinterpret_cast<uintptr_t>(src) + 13u;
    const uint32_t off = static_cast<uint32_t>(ct & 15u);
    const int lq = off == 0 ? 4 : static_cast<int>(off >> 2);
    oa.load_r = off & 3u;

    cudaError_t e;
    switch (lq) {
    case 0: e = launch_open_ghash_t<0>(oa, s); break;
    case 1: e = launch_open_ghash_t<1>(oa, s); break;
    case 2: e = launch_open_ghash_t<2>(oa, s); break;
    case 3: e = launch_open_ghash_t<3>(oa, s); break;
    default: e = launch_open_ghash_t<4>(oa, s); break;
    }
    if (e != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }

    dev::CtrArgs ca{};
    ca.frame = oa.frame;
    ca.frame_len = frame_len;
    ca.dst = static_cast<uint8_t*>(dst);
    ca.plen = plaintext_len;
    ca.nblocks = static_cast<uint32_t>(n);
    ca.load_r = oa.load_r;
    std::memcpy(ca.rk, h->rk, sizeof(ca.rk));
    ca.aes_t = h->kt.aes_t;
    ca.auth_ok = auth_ok;
    const uint64_t want = (n + dev::kCtrThreads - 1) / dev::kCtrThreads;
    const uint32_t grid = static_cast<uint32_t>(want < static_cast<uint64_t>(h->num_sms) ? want : h->num_sms);
    const bool pt_aligned = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
    if (pt_aligned) {
        switch (lq) {
        case 0: e = launch_open_ctr_t<0, true>(ca, grid, s); break;
        case 1: e = launch_open_ctr_t<1, true>(ca, grid, s); break;
        case 2: e = launch_open_ctr_t<2, true>(ca, grid, s); break;
        case 3: e = launch_open_ctr_t<3, true>(ca, grid, s); break;
        default: e = launch_open_ctr_t<4, true>(ca, grid, s); break;
        }
    } else {
        switch (lq) {
        case 0: e = launch_open_ctr_t<0, false>(ca, grid, s); break;
        case 1: e = launch_open_ctr_t<1, false>(ca, grid, s); break;
        case 2: e = launch_open_ctr_t<2, false>(ca, grid, s); break;
        case 3: e = launch_open_ctr_t<3, false>(ca, grid, s); break;
        default: e = launch_open_ctr_t<4, false>(ca, grid, s); break;
        }
    }
    return cuda_rc(e);
}

extern "C" const char* lmcache_gpu_aesgcm_strerror(int rc)
{
    switch (rc) {
    case LMCACHE_GPU_AESGCM_OK:
        return "success";
    case LMCACHE_GPU_AESGCM_ERR_ARGUMENT:
        return "invalid argument";
    case LMCACHE_GPU_AESGCM_ERR_ALLOC:
        return "GPU allocation failure";
    case LMCACHE_GPU_AESGCM_ERR_CUDA:
        return "CUDA failure";
    case LMCACHE_GPU_AESGCM_ERR_INTERNAL:
        return "internal error";
    default:
        return "unknown error";
    }
}
