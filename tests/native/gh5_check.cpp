// Host check of the window GHASH tables (kGhW bits) (test infrastructure, compiled
// by tests/test_clmul.py with g++ together with the product's
// confkv_b200/csrc/host_crypto.cpp): x * M from ghash_table5 and the field
// extraction the kernels use (gh5_field_at7).
#include <cstdint>
#include <cstring>
#include <utility>

#include "gh5.cuh"
#include "host_crypto.h"

namespace {

template <int... G>
void xor_groups(const uint32_t (&w)[4], const uint8_t* tab, uint8_t out[16], std::integer_sequence<int, G...>)
{
    auto one = [&](int g, uint32_t field7) {
        const uint32_t v = (field7 & confkv::kGh5Mask7) >> 7;
        const uint8_t* e = tab + (g * confkv::kGh5Values + v) * 16;
        for (int b = 0; b < 16; ++b) {
            out[b] ^= e[b];
        }
    };
    (one(G, confkv::gh5_field_at7<G>(w)), ...);
}

}  // namespace

extern "C" void gh5_check_mul(const uint8_t* x, const uint8_t* m, uint8_t* out)
{
    static uint8_t tab[confkv::kGh5CompactBytes];
    confkv::ghash_table5(confkv::gf_load(m), tab);
    uint32_t w[4];
    std::memcpy(w, x, 16);
    std::memset(out, 0, 16);
    xor_groups(w, tab, out, std::make_integer_sequence<int, confkv::kGh5Groups>{});
}
