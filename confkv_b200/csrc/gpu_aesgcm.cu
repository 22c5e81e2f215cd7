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
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <utility>

#include "host_common.h"
#include "host_crypto.h"
#include "kernels.cuh"
#include "tiles.cuh"

namespace confkv {
namespace dev {

// Writes the shared-window address at which dynamic shared memory starts for
// a kernel without static shared memory (every kernel with a shared layout is
// one); read once per device by configure_device / noalloc_setup.
__global__ void smem_base_probe_kernel(unsigned int* out)
{
    extern __shared__ __align__(16) uint8_t probe_smem[];
    if (threadIdx.x == 0) {
        out[0] = static_cast<unsigned int>(__cvta_generic_to_shared(probe_smem));
    }
}

// ------------------------------------------------------------ seal kernel
//
// One object, grid = its G tiles (CTA c = tile c, see tiles.cuh). Each thread
// keeps kSealChains GHASH chains (rows r = k mod R, multiplier H^(R*T)) and
// ends with Q_t = sum_r C_r H^(T*(J-1-r)); the CTA's share of GHASH is
// (sum_t Q_t H^(T-1-t)) * H^(d_c), d_c = (G-1-c) J T + 2. The power warp
// computes H^(d_c), E_K(J0) and L*H while the other warps run the rows; the
// last CTA to finish writes the tag.
template <int SQ, bool PT_ALIGNED>
__global__ void __launch_bounds__(kSealThreads, 1) seal_kernel(const SealArgs a)
{
    uint8_t* const smem = layout_smem();
    uint4* part = reinterpret_cast<uint4*>(smem + kSealPart);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    pdl_release();
    fill_aes_smem(smem + kSealAes, a.kt.aes_t);
    fill_gh_smem(smem + kSealGh, a.kt.gh_pow2 + kSealChainLog2 * 512);
    fill_smem<kSealFoldSmemLevels * 512>(reinterpret_cast<uint4*>(smem + kSealFold), a.kt.gh_pow2);
    pdl_wait();
    if (blockIdx.x == 0 && tid == 0) {
        a.frame[0] = 1;
        for (int b = 0; b < 12; ++b) {
            a.frame[1 + b] = static_cast<uint8_t>(a.ivw[b >> 2] >> (8 * (b & 3)));
        }
    }
    __syncthreads();

    const uint64_t P = a.plen;
    const int64_t span = static_cast<int64_t>(a.iters) * kHornerThreads;
    uint8_t* ct = a.frame + 13;

    unsigned long long uhi = 0, ulo = 0;  // power warp: U_p = H^(d_c) * x^(4p)
    uint4 ej0 = make_uint4(0, 0, 0, 0);   // power warp: E_K(J0)
    uint4 lh = make_uint4(0, 0, 0, 0);    // power warp: length block * H

    if (warp == kPowerWarp) {
        const unsigned long long d = static_cast<unsigned long long>(a.grid - 1 - blockIdx.x) *
                                         static_cast<unsigned long long>(span) + 2ull;
        seal_power<true>(a.ivw, a.rk, P, d, a.kt.gh_pow2, lane, ej0, lh, uhi, ulo);
    } else {
        const SealTile t{a.src, ct, P,
                         static_cast<int64_t>(a.nblocks) - static_cast<int64_t>(a.grid - blockIdx.x) * span,
                         static_cast<int64_t>(a.iters),
                         {a.ivw[0] ^ a.rk[0], a.ivw[1] ^ a.rk[1], a.ivw[2] ^ a.rk[2]},
                         a.store_r};
        part[tid] = seal_rows<SQ, PT_ALIGNED>(t, a.rk, a.kt.gh_pow2, tid, lane);
    }
    __syncthreads();
    seal_fold(smem, part, a.kt.gh_pow2, tid);

    if (warp == kPowerWarp) {
        unsigned long long shi, slo;
        if (cta_accumulate(a.slot, part[0], uhi, ulo, lane, a.grid, shi, slo)) {
            const uint4 tag = xor4(xor4(be_to_raw(shi, slo), lh), ej0);
            if (lane < 16) {
                ct[P + lane] = static_cast<uint8_t>(byte_of(tag, lane));
            }
        }
    }
}

// CTR pass of the per-object two-pass seal: the tiles of seal_kernel,
// encryption and ciphertext stores only (no GHASH chain, no power warp, so
// 16 warps of up to 128 registers); CTA 0 writes the header. The GHASH pass
// (open_ghash_kernel<LQ, true, true>) follows on the stream.
template <int SQ, bool PT_ALIGNED>
__global__ void __launch_bounds__(kCtrThreads, 1) seal_ctr_kernel(const SealArgs a)
{
    uint8_t* const smem = layout_smem();
    const int tid = threadIdx.x;
    pdl_release();
    fill_aes_smem(smem + kSealAes, a.kt.aes_t);
    pdl_wait();
    if (blockIdx.x == 0 && tid == 0) {
        a.frame[0] = 1;
        for (int b = 0; b < 12; ++b) {
            a.frame[1 + b] = static_cast<uint8_t>(a.ivw[b >> 2] >> (8 * (b & 3)));
        }
    }
    __syncthreads();
    const int64_t span = static_cast<int64_t>(a.iters) * kHornerThreads;
    const SealTile tile{a.src, a.frame + 13, a.plen,
                        static_cast<int64_t>(a.nblocks) - static_cast<int64_t>(a.grid - blockIdx.x) * span,
                        static_cast<int64_t>(a.iters),
                        {a.ivw[0] ^ a.rk[0], a.ivw[1] ^ a.rk[1], a.ivw[2] ^ a.rk[2]},
                        a.store_r};
    (void)seal_rows<SQ, PT_ALIGNED, false>(tile, a.rk, a.kt.gh_pow2, tid, tid & 31);
}

// Zero-length seal: header + tag = E_K(J0) (GHASH of nothing is 0).
__global__ void seal_empty_kernel(const SealArgs a)
{
    pdl_release();
    pdl_wait();
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
// Same tiles as seal_kernel over the ciphertext at frame + 13, with the
// chains of OpenLayout<WIN> (kernels.cuh). The two-stage fold of the batched
// kernels (tiles.cuh) needs one barrier here: each row warp folds its
// partials with levels 0..3 (shared tables) and hands two values to the
// power warp, which folds them with levels 4..8 (shared or the key's global
// tables). (Seal keeps the block fold: its levels 4..8 would read the key's
// global tables, five dependent L2 round trips that cost 2 MiB objects
// 14 %.) The power warp computes E_K(J0) and L*H up front; the last CTA
// compares the expected tag with the frame's (16 bytes, OR-accumulated) and
// checks the version byte, then writes *auth_ok; with SEAL (the GHASH pass
// of the two-pass seal, frame = the sealed frame) it writes the tag.
template <int LQ, bool WIN, bool SEAL = false>
__global__ void __launch_bounds__(kSealThreads, 1) open_ghash_kernel(const OpenArgs a)
{
    using L = OpenLayout<WIN>;
    uint8_t* const smem = layout_smem();
    uint4* part = reinterpret_cast<uint4*>(smem + L::kPart);  // the row warps' fold values V_0..V_31
    const uint4* fold_tabs = reinterpret_cast<const uint4*>(smem + L::kFold);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    pdl_release();
    if constexpr (WIN) {
        fill_gh5_smem(smem + L::kGh, a.kt.gh_chain5);
    } else {
        fill_gh_smem(smem + L::kGh, a.kt.gh_pow2 + kOpenChainLog2 * 512);
    }
    fill_smem<L::kFoldSmemLevels * 512>(reinterpret_cast<uint4*>(smem + L::kFold), a.kt.gh_pow2);  // H^(2^l)
    fill_smem<512>(reinterpret_cast<uint4*>(smem + L::kHt), a.kt.gh_pow2 + kFoldLevels * 512);      // H^512
    if constexpr (!WIN) {
        fill_smem<256>(reinterpret_cast<uint4*>(smem + L::kAesC), reinterpret_cast<const uint4*>(a.kt.aes_t));
    }
    pdl_wait();
    __syncthreads();

    const uint64_t P = a.plen;
    const int64_t span = static_cast<int64_t>(a.iters) * kHornerThreads;

    unsigned long long uhi = 0, ulo = 0;
    uint4 ej0 = make_uint4(0, 0, 0, 0);
    uint4 lh = make_uint4(0, 0, 0, 0);

    if (warp == kPowerWarp) {
        const unsigned long long d = static_cast<unsigned long long>(a.grid - 1 - blockIdx.x) *
                                         static_cast<unsigned long long>(span) + 2ull;
        const uint32_t* aes_c = WIN ? a.kt.aes_t : reinterpret_cast<const uint32_t*>(smem + L::kAesC);
        open_power<true, !WIN>(a.frame, aes_c, a.rk, P, d, a.kt.gh_pow2, lane, ej0, lh, uhi, ulo);
    } else {
        const OpenTile t{a.frame, a.frame_len, P,
                         static_cast<int64_t>(a.nblocks) - static_cast<int64_t>(a.grid - blockIdx.x) * span,
                         static_cast<int64_t>(a.iters), a.load_r};
        const uint4 q = open_ghash_rows<LQ, L::kChains, L::kAluChains, L::kStepRows, WIN, L::kGh>(
            t, reinterpret_cast<const uint4*>(smem + L::kHt), &a.cm, tid, lane);
        const uint4 v = warp_fold_pairs<false>(q, fold_tabs, lane);
        if (lane < 2) {
            part[2 * warp + lane] = v;
        }
    }
    __syncthreads();

    if (warp == kPowerWarp) {
        const uint4* t4 = (L::kFoldSmemLevels == kFoldLevels ? fold_tabs : a.kt.gh_pow2) + 4 * 512;
        const uint4 fold = power_fold(part[lane], t4, lane);
        unsigned long long shi, slo;
        if (cta_accumulate(a.slot, fold, uhi, ulo, lane, a.grid, shi, slo)) {
            if constexpr (SEAL) {
                const uint4 tag = xor4(xor4(be_to_raw(shi, slo), lh), ej0);
                if (lane < 16) {
                    a.tag_out[13 + P + lane] = static_cast<uint8_t>(byte_of(tag, lane));
                }
            } else if (lane == 0) {
                *a.auth_ok = open_verdict(a.frame, P, shi, slo, lh, ej0);
            }
        }
    }
}

// Zero-length open: only the version byte and tag = E_K(J0) to check.
__global__ void open_empty_kernel(const OpenArgs a)
{
    pdl_release();
    pdl_wait();
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
// zero-filled and no keystream is produced. CTA c owns rows
// [c R, (c+1) R) of kCtrThreads blocks (block i = row*T + thread).
template <int LQ, bool PT_ALIGNED>
__global__ void __launch_bounds__(kCtrThreads, 1) open_ctr_kernel(const CtrArgs a)
{
    uint8_t* const smem = layout_smem();
    constexpr int64_t T = kCtrThreads;
    const int tid = threadIdx.x;
    const int64_t row_begin = static_cast<int64_t>(blockIdx.x) * a.rows_per_cta;
    const int64_t rows_total = (static_cast<int64_t>(a.nblocks) + T - 1) / T;
    int64_t row_end = row_begin + a.rows_per_cta;
    row_end = row_end > rows_total ? rows_total : row_end;

    pdl_release();
    fill_aes_smem(smem, a.aes_t);
    pdl_wait();
    const int ok = *reinterpret_cast<const volatile int*>(a.auth_ok);
    CtrTile t{a.frame, a.frame_len, a.dst, a.plen, row_begin * T, row_end - row_begin, {0u, 0u, 0u}, a.load_r};
    if (!ok) {
        ctr_zero_rows<PT_ALIGNED>(t, tid);
        return;
    }
    __syncthreads();

    const uint4 iv = load_bytes(a.frame + 1, 12);
    t.s012[0] = iv.x ^ a.rk[0];
    t.s012[1] = iv.y ^ a.rk[1];
    t.s012[2] = iv.z ^ a.rk[2];
    ctr_rows<LQ, PT_ALIGNED>(t, a.rk, tid, tid & 31);
}

}  // namespace dev
}  // namespace confkv

// ====================================================================== host

namespace {

using confkv::Gf128;
namespace dev = confkv::dev;
using namespace confkv::host;

// Host-side fault injection for tests: CONFKV_B200_FAIL_ALLOC=1 makes
// key_create report an allocation failure before touching the device.
bool alloc_fault_injected()
{
    const char* v = std::getenv("CONFKV_B200_FAIL_ALLOC");
    return v != nullptr && v[0] == '1';
}

}  // namespace

namespace {
// Window address of dynamic shared memory as the probe read it (-1: not yet).
std::atomic<int64_t> g_window_base{-1};
}  // namespace

uint32_t confkv::host::layout_pad()
{
    const int64_t b = g_window_base.load(std::memory_order_acquire);
    return b < 0 ? 0u : dev::kSmemLayoutBase - static_cast<uint32_t>(b);
}

bool confkv::host::record_layout_base(unsigned int window_base)
{
    if (window_base > dev::kSmemLayoutBase || (window_base & 15u) != 0) {
        return false;
    }
    int64_t expected = -1;
    if (g_window_base.compare_exchange_strong(expected, static_cast<int64_t>(window_base),
                                              std::memory_order_acq_rel)) {
        return true;
    }
    return expected == static_cast<int64_t>(window_base);
}

// Opt every kernel instantiation into its dynamic shared memory once per device.
cudaError_t confkv::host::configure_device(int device)
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
        // Where dynamic shared memory starts on this device decides the gap
        // each launch requests before the kernels' layouts (layout_pad).
        {
            unsigned int* d = nullptr;
            unsigned int base = 0;
            chk(cudaMalloc(&d, sizeof(unsigned int)));
            if (e == cudaSuccess) {
                dev::smem_base_probe_kernel<<<1, 32, 1024>>>(d);
                chk(cudaGetLastError());
                chk(cudaMemcpy(&base, d, sizeof(base), cudaMemcpyDeviceToHost));
                cudaFree(d);
                if (e == cudaSuccess && !record_layout_base(base)) {
                    e = cudaErrorNotSupported;
                }
            }
        }
        chk(allow_smem(dev::seal_kernel<0, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<0, true>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<1, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<1, true>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<2, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<2, true>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<3, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<3, true>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<4, true>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<4, true>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<0, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<0, false>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<1, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<1, false>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<2, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<2, false>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<3, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<3, false>, dev::kCtrSmem));
        chk(allow_smem(dev::seal_kernel<4, false>, dev::kSealSmem));
        chk(allow_smem(dev::seal_ctr_kernel<4, false>, dev::kCtrSmem));
        chk(allow_smem(dev::open_ghash_kernel<0, false>, dev::OpenLayout<false>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<0, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<0, true, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<1, false>, dev::OpenLayout<false>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<1, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<1, true, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<2, false>, dev::OpenLayout<false>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<2, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<2, true, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<3, false>, dev::OpenLayout<false>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<3, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<3, true, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<4, false>, dev::OpenLayout<false>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<4, true>, dev::OpenLayout<true>::kSmem));
        chk(allow_smem(dev::open_ghash_kernel<4, true, true>, dev::OpenLayout<true>::kSmem));
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
        chk(configure_batch_kernels());
        results[device] = e;
    });
    return results[device];
}

namespace {

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

// The slot of `s` on this handle: the stream's own, assigned on its first
// call; nullptr once kSlots other streams hold one (the call then fails with
// ERR_ALLOC instead of sharing a slot with unordered work).
dev::Slot* take_slot(KeyHandle* h, cudaStream_t s)
{
    std::lock_guard<std::mutex> lock(h->slot_mu);
    const auto it = h->stream_slot.find(s);
    if (it != h->stream_slot.end()) {
        return h->slots + it->second;
    }
    if (h->stream_slot.size() >= static_cast<size_t>(kSlots)) {
        return nullptr;
    }
    const uint32_t k = static_cast<uint32_t>(h->stream_slot.size());
    h->stream_slot.emplace(s, k);
    return h->slots + k;
}

template <int SQ, bool A>
cudaError_t launch_seal_t(const dev::SealArgs& args, cudaStream_t s)
{
    return launch_pdl(dev::seal_kernel<SQ, A>, args.grid, dev::kSealThreads, dev::kSealSmem, s, args);
}

template <int SQ, bool A>
cudaError_t launch_seal_ctr_t(const dev::SealArgs& args, cudaStream_t s)
{
    return launch_pdl(dev::seal_ctr_kernel<SQ, A>, args.grid, dev::kCtrThreads, dev::kCtrSmem, s, args);
}

template <int LQ>
cudaError_t launch_seal_ghash_t(const dev::OpenArgs& args, cudaStream_t s)
{
    return launch_pdl(dev::open_ghash_kernel<LQ, true, true>, args.grid, dev::kSealThreads,
                      dev::OpenLayout<true>::kSmem, s, args);
}

template <int LQ>
cudaError_t launch_open_ghash_t(const dev::OpenArgs& args, cudaStream_t s)
{
    if (args.plen >= dev::kOpenWindowMinBytes) {
        return launch_pdl(dev::open_ghash_kernel<LQ, true>, args.grid, dev::kSealThreads, dev::OpenLayout<true>::kSmem,
                          s, args);
    }
    return launch_pdl(dev::open_ghash_kernel<LQ, false>, args.grid, dev::kSealThreads, dev::OpenLayout<false>::kSmem, s,
                      args);
}

template <int LQ, bool A>
cudaError_t launch_open_ctr_t(const dev::CtrArgs& args, uint32_t grid, cudaStream_t s)
{
    return launch_pdl(dev::open_ctr_kernel<LQ, A>, grid, dev::kCtrThreads, dev::kCtrSmem, s, args);
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
    const cudaError_t ce = configure_device(device);
    if (ce == cudaErrorNotSupported) {
        return LMCACHE_GPU_AESGCM_ERR_INTERNAL;  // unexpected shared-memory layout
    }
    if (ce != cudaSuccess) {
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
    const size_t off_pow2 = kAesT;
    const size_t off_chain = off_pow2 + kTab * confkv::kPow2Tables;
    const size_t off_chain5 = off_chain + kTab;
    const size_t off_slots = off_chain5 + confkv::kGh5CompactBytes;
    const size_t total = off_slots + sizeof(dev::Slot) * kSlots;

    uint8_t* host = new (std::nothrow) uint8_t[total];
    if (host == nullptr) {
        delete h;
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }
    std::memset(host, 0, total);
    confkv::aes_t_tables(reinterpret_cast<uint32_t(*)[256]>(host));
    Gf128 p = H;
    for (int k = 0; k < confkv::kPow2Tables; ++k) {
        confkv::ghash_table(p, host + off_pow2 + kTab * k);
        p = confkv::gf_mul(p, p);
    }
    {
        // the batched GHASH passes' chain multiplier: its 4-bit table and
        // its integer-pipe form
        const Gf128 m = confkv::gf_pow(H, static_cast<uint64_t>(dev::kOpenBatchChains) * dev::kHornerThreads);
        confkv::ghash_table(m, host + off_chain);
        confkv::ghash_table5(m, host + off_chain5);
        uint8_t pb[16];
        uint32_t pw[4];
        confkv::gf_store(pb, m);
        std::memcpy(pw, pb, 16);
        h->open_cm = confkv::clmul_prepare(pw);
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
    h->kt.gh_pow2 = reinterpret_cast<const uint4*>(h->d_mem + off_pow2);
    h->kt.gh_chain = reinterpret_cast<const uint4*>(h->d_mem + off_chain);
    h->kt.gh_chain5 = reinterpret_cast<const uint4*>(h->d_mem + off_chain5);
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

// Large objects: CTR pass (seal_ctr_kernel), then the window-table GHASH
// pass over the frame's ciphertext, which writes the tag; both on the tiles
// and the accumulation slot of `args`.
static int seal_two_pass(const KeyHandle* h, const dev::SealArgs& args, size_t dst_capacity, int sq, bool pt_aligned,
                  cudaStream_t s)
{
    cudaError_t e;
    if (pt_aligned) {
        switch (sq) {
        case 0: e = launch_seal_ctr_t<0, true>(args, s); break;
        case 1: e = launch_seal_ctr_t<1, true>(args, s); break;
        case 2: e = launch_seal_ctr_t<2, true>(args, s); break;
        case 3: e = launch_seal_ctr_t<3, true>(args, s); break;
        default: e = launch_seal_ctr_t<4, true>(args, s); break;
        }
    } else {
        switch (sq) {
        case 0: e = launch_seal_ctr_t<0, false>(args, s); break;
        case 1: e = launch_seal_ctr_t<1, false>(args, s); break;
        case 2: e = launch_seal_ctr_t<2, false>(args, s); break;
        case 3: e = launch_seal_ctr_t<3, false>(args, s); break;
        default: e = launch_seal_ctr_t<4, false>(args, s); break;
        }
    }
    if (e != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    dev::OpenArgs oa{};
    oa.frame = args.frame;
    oa.frame_len = dst_capacity;
    oa.plen = args.plen;
    oa.nblocks = args.nblocks;
    oa.iters = args.iters;
    oa.grid = args.grid;
    std::memcpy(oa.rk, h->rk, sizeof(oa.rk));
    oa.kt = h->kt;
    oa.slot = args.slot;
    oa.cm = h->open_cm;
    oa.tag_out = args.frame;
    const uint32_t off = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(args.frame) + 13u) & 15u);
    const int lq = off == 0 ? 4 : static_cast<int>(off >> 2);
    oa.load_r = off & 3u;
    switch (lq) {
    case 0: e = launch_seal_ghash_t<0>(oa, s); break;
    case 1: e = launch_seal_ghash_t<1>(oa, s); break;
    case 2: e = launch_seal_ghash_t<2>(oa, s); break;
    case 3: e = launch_seal_ghash_t<3>(oa, s); break;
    default: e = launch_seal_ghash_t<4>(oa, s); break;
    }
    std::memset(oa.rk, 0, sizeof(oa.rk));
    return cuda_rc(e);
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
        return cuda_rc(launch_pdl(dev::seal_empty_kernel, 1, 32, 0, s, args));
    }
    horner_grid(n, h->num_sms, args.iters, args.grid);
    args.slot = take_slot(h, s);
    if (args.slot == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }

    const uintptr_t ct = reinterpret_cast<uintptr_t>(dst) + 13u;
    const uint32_t off = static_cast<uint32_t>(ct & 15u);
    const bool pt_aligned = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    int sq = 4;
    if (off != 0) {
        const uint32_t sh = 16u - off;
        sq = static_cast<int>(sh >> 2);
        args.store_r = sh & 3u;
    }
    if (plaintext_len >= dev::kSealTwoPassMinBytes) {
        return seal_two_pass(h, args, dst_capacity, sq, pt_aligned, s);
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
    oa.cm = h->open_cm;

    if (n == 0) {
        return cuda_rc(launch_pdl(dev::open_empty_kernel, 1, 32, 0, s, oa));
    }
    horner_grid(n, h->num_sms, oa.iters, oa.grid);
    oa.slot = take_slot(h, s);
    if (oa.slot == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ALLOC;
    }

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
    const uint64_t rows_total = (n + dev::kCtrThreads - 1) / dev::kCtrThreads;
    const uint64_t sms = static_cast<uint64_t>(h->num_sms);
    const uint64_t rows_per_cta = (rows_total + sms - 1) / sms;
    ca.rows_per_cta = static_cast<uint32_t>(rows_per_cta);
    const uint32_t grid = static_cast<uint32_t>((rows_total + rows_per_cta - 1) / rows_per_cta);
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

// ===================================================== seal without allocation
//
// lmcache_gpu_aes128gcm_seal_noalloc serves callers that cannot call
// cudaMalloc at the point where they seal: a KV-cache server that has handed
// (nearly) all device memory to its own pool at start-up, or a pipeline
// thread that must not hit cudaMalloc's implicit device synchronisation. It
// takes the raw key instead of a handle and keeps everything the seal kernel
// needs beyond its input and output -- the key's GHASH tables, the AES
// T-tables and the call's accumulation slot -- in one file-scope __device__
// array that every GPU loading this library holds until process exit.
//
// Which key's tables the array holds is decided on the device, in stream
// order: every call launches noalloc_prepare_kernel with H = E_K(0^128),
// which compares H with the record kept beside each table and rebuilds only
// the tables built for another key; the seal kernel follows it on the stream.
// The host keeps no key material between calls.
namespace {

constexpr int kNoAllocPow2Tables = 28;  // H^(2^k), k < 28: exponents of objects up to 1 GiB
constexpr size_t kNoAllocAesBytes = 4 * 256 * sizeof(uint32_t);
constexpr size_t kNoAllocTableBytes =
    kNoAllocAesBytes + static_cast<size_t>(kNoAllocPow2Tables) * confkv::kGhashTableBytes;
constexpr size_t kNoAllocRecordOffset = kNoAllocTableBytes;  // 32 B per table: {H, valid word}
constexpr size_t kNoAllocSlotOffset = (kNoAllocRecordOffset + 32 * kNoAllocPow2Tables + 255) / 256 * 256;
constexpr size_t kNoAllocScratchBytes = kNoAllocSlotOffset + 256;
constexpr uint64_t kNoAllocMaxPlaintext = 1ull << 30;
constexpr uint32_t kNoAllocRecordValid = 0x48746162u;

static_assert(dev::kSealChainLog2 < kNoAllocPow2Tables, "chain multiplier table must be in the scratch");

// The shared scratch array (229,376 B + 1,024 B of table records and slot per device).
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// One warp per GHASH table t (H^(2^t)), one CTA. A warp whose record names
// `h` leaves its table alone; otherwise it forms H^(2^t) by t squarings,
// rebuilds the 4-bit table (lane L holds U_L = H^(2^t) x^(4L) and writes the
// 16 entries of nibble position L ^ 1, see ghash_table in host_crypto.cpp)
// and then rewrites the record. Warp 0 also clears the accumulation slot.
__global__ void __launch_bounds__(32 * kNoAllocPow2Tables) noalloc_prepare_kernel(uint8_t* scratch, const uint4 h)
{
    const int lane = static_cast<int>(threadIdx.x & 31u);
    const int t = static_cast<int>(threadIdx.x >> 5);
    if (threadIdx.x == 0) {
        auto* slot = reinterpret_cast<dev::Slot*>(scratch + kNoAllocSlotOffset);
        slot->acc_hi = 0;
        slot->acc_lo = 0;
        slot->ticket = 0;
    }
    uint4* rec = reinterpret_cast<uint4*>(scratch + kNoAllocRecordOffset + 32 * static_cast<size_t>(t));
    const uint4 have = rec[0];
    if (rec[1].x == kNoAllocRecordValid && have.x == h.x && have.y == h.y && have.z == h.z && have.w == h.w) {
        return;
    }
    uint4 m = h;
    for (int k = 0; k < t; ++k) {
        unsigned long long uhi, ulo, rhi, rlo;
        dev::warp_lane_basis(m, lane, uhi, ulo);
        dev::warp_generic_mul(m, uhi, ulo, lane, rhi, rlo);
        m = dev::be_to_raw(rhi, rlo);
    }
    unsigned long long bh[4], bl[4];  // B_c = U_L x^(3-c): the product for nibble bit c
    dev::warp_lane_basis(m, lane, bh[3], bl[3]);
    for (int c = 2; c >= 0; --c) {
        bh[c] = bh[c + 1];
        bl[c] = bl[c + 1];
        dev::gf_mul_x(bh[c], bl[c]);
    }
    uint4* tab = reinterpret_cast<uint4*>(scratch + kNoAllocAesBytes + static_cast<size_t>(t) * confkv::kGhashTableBytes) +
                 16 * (lane ^ 1);
    for (int v = 0; v < 16; ++v) {
        unsigned long long eh = 0, el = 0;
        for (int c = 0; c < 4; ++c) {
            if ((v >> c) & 1) {
                eh ^= bh[c];
                el ^= bl[c];
            }
        }
        tab[v] = dev::be_to_raw(eh, el);
    }
    __syncwarp();
    if (lane == 0) {
        rec[0] = h;
        rec[1] = make_uint4(kNoAllocRecordValid, 0u, 0u, 0u);
    }
}

struct NoAllocDevice {
    std::once_flag once;
    int status = LMCACHE_GPU_AESGCM_OK;
    uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int num_sms = 0;
    std::mutex mu;               // keeps a call's prepare and seal launches adjacent on a stream
};

NoAllocDevice g_noalloc_dev[kMaxDevices];

// Once per device, with that device current: resolve the array's device
// address, read where dynamic shared memory starts (the probe kernel writes
// into the array), opt the seal kernels into their shared memory and copy in
// the key-independent AES T-tables. Synchronous; allocates nothing.
int noalloc_setup(int device, NoAllocDevice& st)
{
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&st.scratch), g_noalloc_scratch) != cudaSuccess ||
        st.scratch == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    if (cudaDeviceGetAttribute(&st.num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        st.num_sms <= 0) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    // The seal kernels' launches request the gap before their shared layout
    // (layout_pad), so where dynamic shared memory starts is read first.
    unsigned int* probe = reinterpret_cast<unsigned int*>(st.scratch + kNoAllocSlotOffset + 128);
    dev::smem_base_probe_kernel<<<1, 32, 1024>>>(probe);
    unsigned int base = 0;
    if (cudaGetLastError() != cudaSuccess ||
        cudaMemcpy(&base, probe, sizeof(base), cudaMemcpyDeviceToHost) != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    if (!record_layout_base(base)) {
        return LMCACHE_GPU_AESGCM_ERR_INTERNAL;
    }
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
    if (e != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    uint32_t aes_t[4][256];
    confkv::aes_t_tables(aes_t);
    if (cudaMemcpy(st.scratch, aes_t, kNoAllocAesBytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    return LMCACHE_GPU_AESGCM_OK;
}

// Plain (not programmatic) launch: the kernel starts only after everything
// before it on the stream, the prepare kernel's table writes included, has
// completed.
template <int SQ, bool A>
cudaError_t launch_seal_plain(const dev::SealArgs& args, cudaStream_t s)
{
    dev::seal_kernel<SQ, A><<<args.grid, dev::kSealThreads, launch_smem(dev::kSealSmem), s>>>(args);
    return cudaGetLastError();
}

}  // namespace

extern "C" int lmcache_gpu_aes128gcm_seal_noalloc(const uint8_t* key, size_t key_len, const void* src,
                                                  size_t plaintext_len, void* dst, size_t dst_capacity,
                                                  const uint8_t* iv, int device, void* stream_ptr)
{
    if (key == nullptr || key_len != 16 || src == nullptr || dst == nullptr || iv == nullptr) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    if (plaintext_len > kNoAllocMaxPlaintext ||
        dst_capacity < lmcache_gpu_aesgcm_frame_size(plaintext_len)) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    if (device < 0 || device >= kMaxDevices) {
        return LMCACHE_GPU_AESGCM_ERR_ARGUMENT;
    }
    DeviceGuard guard(device);
    if (!guard.ok()) {
        return LMCACHE_GPU_AESGCM_ERR_CUDA;
    }
    NoAllocDevice& st = g_noalloc_dev[device];
    std::call_once(st.once, [&]() { st.status = noalloc_setup(device, st); });
    if (st.status != LMCACHE_GPU_AESGCM_OK) {
        return st.status;
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream_ptr);

    dev::SealArgs args{};
    args.src = static_cast<const uint8_t*>(src);
    args.frame = static_cast<uint8_t*>(dst);
    args.plen = plaintext_len;
    const uint64_t n = (static_cast<uint64_t>(plaintext_len) + 15u) / 16u;
    args.nblocks = static_cast<uint32_t>(n);
    for (int k = 0; k < 3; ++k) {
        args.ivw[k] = le_word(iv + 4 * k);
    }
    confkv::aes128_expand_le(key, args.rk);
    args.kt.aes_t = reinterpret_cast<const uint32_t*>(st.scratch);
    args.kt.gh_pow2 = reinterpret_cast<const uint4*>(st.scratch + kNoAllocAesBytes);
    args.slot = reinterpret_cast<dev::Slot*>(st.scratch + kNoAllocSlotOffset);

    cudaError_t e;
    if (n == 0) {
        // header + E_K(J0): reads only the key-independent T-tables
        args.grid = 1;
        dev::seal_empty_kernel<<<1, 32, 0, s>>>(args);
        e = cudaGetLastError();
        std::memset(args.rk, 0, sizeof(args.rk));
        return cuda_rc(e);
    }
    uint8_t zero[16] = {0};
    uint8_t hbytes[16];
    confkv::aes128_encrypt_block(args.rk, zero, hbytes);
    uint4 h;
    std::memcpy(&h, hbytes, 16);
    std::memset(hbytes, 0, sizeof(hbytes));

    horner_grid(n, st.num_sms, args.iters, args.grid);
    const uintptr_t ct = reinterpret_cast<uintptr_t>(dst) + 13u;
    const uint32_t off = static_cast<uint32_t>(ct & 15u);
    const bool pt_aligned = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    int sq = 4;
    if (off != 0) {
        const uint32_t sh = 16u - off;
        sq = static_cast<int>(sh >> 2);
        args.store_r = sh & 3u;
    }
    {
        // Two host threads sharing a stream must not interleave their
        // prepare and seal launches (the second prepare would swap the tables
        // under the first seal).
        std::lock_guard<std::mutex> lock(st.mu);
        noalloc_prepare_kernel<<<1, 32 * kNoAllocPow2Tables, 0, s>>>(st.scratch, h);
        e = cudaGetLastError();
        if (e == cudaSuccess) {
            if (pt_aligned) {
                switch (sq) {
                case 0: e = launch_seal_plain<0, true>(args, s); break;
                case 1: e = launch_seal_plain<1, true>(args, s); break;
                case 2: e = launch_seal_plain<2, true>(args, s); break;
                case 3: e = launch_seal_plain<3, true>(args, s); break;
                default: e = launch_seal_plain<4, true>(args, s); break;
                }
            } else {
                switch (sq) {
                case 0: e = launch_seal_plain<0, false>(args, s); break;
                case 1: e = launch_seal_plain<1, false>(args, s); break;
                case 2: e = launch_seal_plain<2, false>(args, s); break;
                case 3: e = launch_seal_plain<3, false>(args, s); break;
                default: e = launch_seal_plain<4, false>(args, s); break;
                }
            }
        }
    }
    std::memset(&h, 0, sizeof(h));
    std::memset(args.rk, 0, sizeof(args.rk));
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
