// Issue-rate microbenchmark of the integer and shared-memory instructions the
// seal/open kernels are built from, on this GPU. It supplies the measured
// peaks of the integer roofline (bench.py) and of the shared-memory
// wavefront bound; it is a measurement, not part of the seal/open C-ABI.
//
//   int pipe_rates_run(int op, int iters, double* per_sm_clk, double* cycles)
//
// launches one CTA of 1024 threads per SM; every thread runs `iters`
// iterations of kChains x kUnroll independent instructions of kind `op`
// (kChains dependency chains, so issue, not latency, binds). CTA c reads
// %clock64 around its loop (after a barrier on both sides). Returns, in
// *per_sm_clk, the instructions of that kind executed per SM per SM clock,
// counted in threads (a 32-lane warp instruction counts 32), averaged over
// CTAs, and in *cycles the mean loop cycles. ops: see PipeOp.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

enum PipeOp : int {
    kLop3 = 0,      // lop3.b32 (xor of three)
    kIadd = 1,      // add.u32 (ptxas merges two dependent adds into one IADD3: per IADD3, half this rate)
    kPrmt = 2,      // prmt.b32 with a register selector
    kShf = 3,       // shf.l.wrap.b32
    kImad = 4,      // mad.lo.u32
    kImadWide = 5,  // mad.wide.u32 (32 x 32 + 64 -> 64)
    kImadHi = 6,    // mul.hi.u32
    kLds32 = 7,     // ld.shared.u32, 32 lanes on 32 banks (one wavefront)
    kLds128 = 8,    // ld.shared.v4.u32, 32 lanes x 16 B (four wavefronts)
    kMixed = 9,     // lop3.b32 on half the chains, mad.lo.u32 on the other half (ALU and FMA pipes: issue rate)
    kShfl = 10,     // shfl.sync.idx.b32 from lane ^ 1
    kLdsShfl = 11,  // ld.shared.u32 (one wavefront) on half the chains, shfl.sync on the other half
    kOps = 12,
};

constexpr int kThreads = 1024;
constexpr int kChains = 8;
constexpr int kUnroll = 16;

template <int OP>
__device__ __forceinline__ void step(uint32_t (&x)[kChains], unsigned long long (&w)[kChains], uint32_t a,
                                     uint32_t b, uint32_t s32, uint32_t s128, uint32_t src_lane)
{
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
        if constexpr (OP == kLop3) {
            asm volatile("lop3.b32 %0, %0, %1, %2, 0x96;" : "+r"(x[c]) : "r"(a), "r"(b));
        } else if constexpr (OP == kIadd) {
            asm volatile("add.u32 %0, %0, %1;" : "+r"(x[c]) : "r"(a));
        } else if constexpr (OP == kPrmt) {
            asm volatile("prmt.b32 %0, %0, %1, %2;" : "+r"(x[c]) : "r"(a), "r"(b));
        } else if constexpr (OP == kShf) {
            asm volatile("shf.l.wrap.b32 %0, %0, %1, %2;" : "+r"(x[c]) : "r"(a), "r"(b));
        } else if constexpr (OP == kImad) {
            asm volatile("mad.lo.u32 %0, %0, %1, %2;" : "+r"(x[c]) : "r"(a), "r"(b));
        } else if constexpr (OP == kImadWide) {
            // the multiplicand is the accumulator's low word, so no product can be hoisted
            asm volatile("{\n\t.reg .u32 lo;\n\tcvt.u32.u64 lo, %0;\n\tmad.wide.u32 %0, lo, %1, %0;\n\t}"
                         : "+l"(w[c])
                         : "r"(b));
        } else if constexpr (OP == kImadHi) {
            asm volatile("mul.hi.u32 %0, %0, %1;" : "+r"(x[c]) : "r"(a));
        } else if constexpr (OP == kMixed) {
            if (c & 1) {
                asm volatile("mad.lo.u32 %0, %0, %1, %2;" : "+r"(x[c]) : "r"(a), "r"(b));
            } else {
                asm volatile("lop3.b32 %0, %0, %1, %2, 0x96;" : "+r"(x[c]) : "r"(a), "r"(b));
            }
        } else if (OP == kShfl || (OP == kLdsShfl && (c & 1))) {  // c is unrolled: folds at compile time
            asm volatile("shfl.sync.idx.b32 %0, %0, %1, 31, 0xffffffff;" : "+r"(x[c]) : "r"(src_lane));
        } else if constexpr (OP == kLds32 || OP == kLdsShfl) {
            uint32_t v;
            asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(s32 + 128u * static_cast<uint32_t>(c)));
            x[c] ^= v;
        } else {
            uint32_t v0, v1, v2, v3;
            asm volatile("ld.volatile.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                         : "r"(s128 + 512u * static_cast<uint32_t>(c)));
            x[c] ^= v0 ^ v1 ^ v2 ^ v3;
        }
    }
}

template <int OP>
__global__ void __launch_bounds__(kThreads, 1) pipe_kernel(int iters, unsigned long long* cycles, uint32_t* sink)
{
    __shared__ __align__(16) uint32_t tab[4 * kThreads];
    for (int i = threadIdx.x; i < 4 * kThreads; i += kThreads) {
        tab[i] = static_cast<uint32_t>(i) * 2654435761u;
    }
    const uint32_t lane = threadIdx.x & 31u;
    // lane l reads word l of a 128-byte row (LDS.32) or 16-byte slot l of a
    // 512-byte row (LDS.128): conflict-free; every address stays inside tab
    // (at most 16 * 31 + 512 * 7 + 16 = 4,096 of its 16,384 bytes)
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(tab));
    const uint32_t s32 = sbase + 4u * lane;
    const uint32_t s128 = sbase + 16u * lane;
    uint32_t x[kChains];
    unsigned long long w[kChains];
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
        x[c] = threadIdx.x * 0x9e3779b9u + static_cast<uint32_t>(c);
        w[c] = x[c];
    }
    const uint32_t a = sink[0] | 0x01234567u;  // runtime values the compiler cannot fold
    const uint32_t b = sink[1] | 0x00000101u;
    __syncthreads();
    const unsigned long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            step<OP>(x, w, a, b, s32, s128, lane ^ 1u);
        }
    }
    __syncthreads();
    const unsigned long long t1 = clock64();
    uint32_t r = 0;
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
        r ^= x[c] ^ static_cast<uint32_t>(w[c]) ^ static_cast<uint32_t>(w[c] >> 32);
    }
    if (r == 0x5eed5eedu) {
        sink[2 + (threadIdx.x & 7)] = r;  // keeps the chains live
    }
    if (threadIdx.x == 0) {
        cycles[blockIdx.x] = t1 - t0;
    }
}

template <int OP>
cudaError_t launch(int sms, int iters, unsigned long long* cycles, uint32_t* sink)
{
    pipe_kernel<OP><<<sms, kThreads>>>(iters, cycles, sink);
    return cudaGetLastError();
}

}  // namespace

extern "C" int pipe_rates_run(int op, int iters, double* per_sm_clk, double* mean_cycles)
{
    if (op < 0 || op >= kOps || iters <= 0 || per_sm_clk == nullptr || mean_cycles == nullptr) {
        return -1;
    }
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
        return -3;
    }
    unsigned long long* d_cycles = nullptr;
    uint32_t* d_sink = nullptr;
    if (cudaMalloc(&d_cycles, sizeof(unsigned long long) * static_cast<size_t>(sms)) != cudaSuccess) {
        return -2;
    }
    if (cudaMalloc(&d_sink, 64) != cudaSuccess || cudaMemset(d_sink, 0, 64) != cudaSuccess) {
        cudaFree(d_cycles);
        return -2;
    }
    cudaError_t e = cudaSuccess;
    for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {  // the first run warms up
        switch (op) {
        case kLop3: e = launch<kLop3>(sms, iters, d_cycles, d_sink); break;
        case kIadd: e = launch<kIadd>(sms, iters, d_cycles, d_sink); break;
        case kPrmt: e = launch<kPrmt>(sms, iters, d_cycles, d_sink); break;
        case kShf: e = launch<kShf>(sms, iters, d_cycles, d_sink); break;
        case kImad: e = launch<kImad>(sms, iters, d_cycles, d_sink); break;
        case kImadWide: e = launch<kImadWide>(sms, iters, d_cycles, d_sink); break;
        case kImadHi: e = launch<kImadHi>(sms, iters, d_cycles, d_sink); break;
        case kLds32: e = launch<kLds32>(sms, iters, d_cycles, d_sink); break;
        case kLds128: e = launch<kLds128>(sms, iters, d_cycles, d_sink); break;
        case kShfl: e = launch<kShfl>(sms, iters, d_cycles, d_sink); break;
        case kLdsShfl: e = launch<kLdsShfl>(sms, iters, d_cycles, d_sink); break;
        default: e = launch<kMixed>(sms, iters, d_cycles, d_sink); break;
        }
        if (e == cudaSuccess) {
            e = cudaDeviceSynchronize();
        }
    }
    int rc = e == cudaSuccess ? 0 : -3;
    if (rc == 0) {
        unsigned long long* h = new unsigned long long[static_cast<size_t>(sms)];
        if (cudaMemcpy(h, d_cycles, sizeof(unsigned long long) * static_cast<size_t>(sms), cudaMemcpyDeviceToHost) !=
            cudaSuccess) {
            rc = -3;
        } else {
            const double ops = static_cast<double>(kThreads) * iters * kUnroll * kChains;
            double rate = 0.0, cyc = 0.0;
            for (int c = 0; c < sms; ++c) {
                rate += ops / static_cast<double>(h[c]);
                cyc += static_cast<double>(h[c]);
            }
            *per_sm_clk = rate / sms;
            *mean_cycles = cyc / sms;
        }
        delete[] h;
    }
    cudaFree(d_cycles);
    cudaFree(d_sink);
    return rc;
}
