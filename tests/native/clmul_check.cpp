// Host build of confkv_b200/csrc/clmul.cuh for the CPU tests (test
// infrastructure, compiled by tests/test_clmul.py with g++): exposes the
// integer-pipe GF(2^128) multiply and a GHASH Horner chain over it.
#include <cstddef>
#include <cstdint>
#include <cstring>

#include "clmul.cuh"

extern "C" void clmul_check_mul(const uint8_t* a, const uint8_t* m, uint8_t* out, int h5)
{
    uint32_t ar[4], mr[4], x[4], y[4], raw[4];
    std::memcpy(ar, a, 16);
    std::memcpy(mr, m, 16);
    const confkv::ClmulConst c = confkv::clmul_prepare(mr);
    confkv::clmul_from_raw(ar, x);
    if (h5) {
        confkv::clmul_mul_int<true>(x, c, y);
    } else {
        confkv::clmul_mul_int<false>(x, c, y);
    }
    confkv::clmul_to_raw(y, raw);
    std::memcpy(out, raw, 16);
}

// sum_i C_i H^(n - i) over n full blocks, by Horner with M = H.
extern "C" void clmul_check_ghash(const uint8_t* h, const uint8_t* data, size_t nblocks, uint8_t* out, int h5)
{
    uint32_t hr[4], acc[4] = {0, 0, 0, 0}, raw[4];
    std::memcpy(hr, h, 16);
    const confkv::ClmulConst c = confkv::clmul_prepare(hr);
    for (size_t i = 0; i < nblocks; ++i) {
        uint32_t blk[4], ci[4];
        std::memcpy(blk, data + 16 * i, 16);
        confkv::clmul_from_raw(blk, ci);
        for (int w = 0; w < 4; ++w) {
            acc[w] ^= ci[w];
        }
        uint32_t t[4];
        if (h5) {
            confkv::clmul_mul_int<true>(acc, c, t);
        } else {
            confkv::clmul_mul_int<false>(acc, c, t);
        }
        std::memcpy(acc, t, sizeof(acc));
    }
    confkv::clmul_to_raw(acc, raw);
    std::memcpy(out, raw, 16);
}
