// GF(2^128) multiplication by a fixed multiplier M on the integer pipes, for
// the GHASH Horner chains that do not use the shared-memory tables. Host and
// device compile the same code (the host prepares M's operands and the CPU
// tests check this file against the bit-serial SP 800-38D multiply).
//
// Field elements: GHASH blocks as four little-endian 32-bit words r[0..3]
// (word c = block bytes 4c..4c+3, byte 4c in the low bits; block bit 0 = the
// MSB of byte 0 = the coefficient of x^0). For the integer arithmetic a block
// is read as the 128-bit integer a = sum_i A_i 2^(127-i) (A_i = coefficient
// of x^i, "reflected"): a's word w (w = 0 least significant) is
// bswap(r[3 - w]).
//
// Carry-less product (T. Pornin's integer-multiply method, written here from
// its published description, with two levels of Karatsuba): a 32 x 32 -> 64
// carry-less product takes the operands' bits at positions = i (mod 4) as
// x_i, y_j, forms the 16 integer products x_i * y_j with IMAD.WIDE, and keeps
// bit 0 of every 4-bit hole of the products whose residues add up to the
// output position: every hole of an integer product holds a count of at most
// 8 (each operand part has 8 bits), so products never carry into the next
// hole and their XOR keeps each hole's parity. 128 x 128 is Karatsuba over
// 64-bit halves, each Karatsuba over 32-bit words: 9 products, 144 IMAD.WIDE.
//
// Reduction: with a and b reflected, the integer carry-less product p
// (255 bits, x^s at bit 254 - s) is the reflected 256-bit form of
// A(x) B(x) x (x^s at bit 255 - s): its high half holds the powers 0..127
// and its low half h the powers 128..255. With x^128 = 1 + x + x^2 + x^7 and
// multiplication by x^k a right shift by k of a reflected value, the powers
// h x^k pushes past x^127 are t = (h << 127) ^ (h << 126) ^ (h << 121)
// (mod 2^128); with g = h ^ t,
//     A B x mod P = p_hi ^ g ^ (g >> 1) ^ (g >> 2) ^ (g >> 7).
// The multiplier is therefore prepared as M x^-1 (x^-1 = x^127 + x^6 + x + 1,
// since x (x^127 + x^6 + x + 1) = x^128 + x^7 + x^2 + x = 1 mod P): the
// product is A M with no shift of p.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define CONFKV_CLMUL_FN __host__ __device__ __forceinline__
#else
#define CONFKV_CLMUL_FN inline
#endif

namespace confkv {

constexpr uint32_t kClmulHole = 0x11111111u;

// Spacing-5 holes (clmul32_h5): x's bits at positions = i (mod 5) and y's
// at = j (mod 5), y restricted to its low 31 bits. For one output residue r
// the five products x_i * y_(r-i) are SUMMED (IMAD.WIDE accumulation, no
// XOR): a hole's count over all five is #{(p, q): p + q = k, p < 32, q < 31}
// <= 31, which fits its 5 bits. y's bit 31 adds x << 31 (a shift).
// Positions = i (mod 5) of a 32-bit word: kClmulH5 << i; of a 64-bit word: kClmulH5w << i.
constexpr uint32_t kClmulH5 = 0x42108421u;
constexpr uint64_t kClmulH5w = 0x1084210842108421ull;

// M prepared for clmul_mul: the 9 Karatsuba operands of M's integer words
// b0..b3 (b0 least significant) -- b0, b1, b0^b1, b2, b3, b2^b3, b0^b2,
// b1^b3, b0^b1^b2^b3 -- each as its 4 holed parts y & (kClmulHole << j)
// (spacing 4), and as its 5 spacing-5 parts of the low 31 bits with bit k of
// top5 = bit 31 of operand k.
struct ClmulConst {
    uint32_t y[9][4];
    uint32_t y5[9][5];
    uint32_t top5;
};

CONFKV_CLMUL_FN uint32_t clmul_bswap(uint32_t x)
{
#if defined(__CUDA_ARCH__)
    return __byte_perm(x, 0, 0x0123);
#else
    return (x >> 24) | ((x >> 8) & 0xff00u) | ((x << 8) & 0xff0000u) | (x << 24);
#endif
}

CONFKV_CLMUL_FN void clmul_parts(uint32_t v, uint32_t out[4])
{
    for (int j = 0; j < 4; ++j) {
        out[j] = v & (kClmulHole << j);
    }
}

// Host: M (raw block words) -> the Karatsuba operands of M x^-1. In the
// reflected integer form, M x^-1 = (M << 1), plus x^-1 = x^127 + x^6 + x + 1
// when the shift pushes out M's x^0 coefficient (bit 127).
CONFKV_CLMUL_FN ClmulConst clmul_prepare(const uint32_t m_raw[4])
{
    uint32_t b[4];  // M's integer words, b[0] least significant
    for (int w = 0; w < 4; ++w) {
        b[w] = clmul_bswap(m_raw[3 - w]);
    }
    const uint32_t carry = b[3] >> 31;  // M's coefficient of x^0
    for (int w = 3; w > 0; --w) {
        b[w] = (b[w] << 1) | (b[w - 1] >> 31);
    }
    b[0] <<= 1;
    // x^-1 reflected: x^0 at bit 127, x^1 at 126, x^6 at 121, x^127 at 0
    const uint32_t xinv[4] = {0x00000001u, 0u, 0u, 0xC2000000u};
    for (int w = 0; w < 4; ++w) {
        b[w] ^= carry * xinv[w];
    }
    const uint32_t b0 = b[0], b1 = b[1], b2 = b[2], b3 = b[3];
    const uint32_t ops[9] = {b0, b1, b0 ^ b1, b2, b3, b2 ^ b3, b0 ^ b2, b1 ^ b3, b0 ^ b1 ^ b2 ^ b3};
    ClmulConst c{};
    for (int k = 0; k < 9; ++k) {
        clmul_parts(ops[k], c.y[k]);
        for (int j = 0; j < 5; ++j) {
            c.y5[k][j] = ops[k] & 0x7fffffffu & (kClmulH5 << j);
        }
        c.top5 |= (ops[k] >> 31) << k;
    }
    return c;
}

// 32 x 32 -> 64 carry-less product with spacing-5 holes; y as its 5 parts
// of the low 31 bits, `top` = y's bit 31.
CONFKV_CLMUL_FN uint64_t clmul32_h5(uint32_t x, const uint32_t y[5], bool top)
{
    const uint64_t x0 = x & kClmulH5, x1 = x & (kClmulH5 << 1), x2 = x & (kClmulH5 << 2);
    const uint64_t x3 = x & (kClmulH5 << 3), x4 = x & (kClmulH5 << 4);
    const uint64_t y0 = y[0], y1 = y[1], y2 = y[2], y3 = y[3], y4 = y[4];
    const uint64_t z0 = x0 * y0 + x1 * y4 + x2 * y3 + x3 * y2 + x4 * y1;
    const uint64_t z1 = x0 * y1 + x1 * y0 + x2 * y4 + x3 * y3 + x4 * y2;
    const uint64_t z2 = x0 * y2 + x1 * y1 + x2 * y0 + x3 * y4 + x4 * y3;
    const uint64_t z3 = x0 * y3 + x1 * y2 + x2 * y1 + x3 * y0 + x4 * y4;
    const uint64_t z4 = x0 * y4 + x1 * y3 + x2 * y2 + x3 * y1 + x4 * y0;
    uint64_t r = (z0 & kClmulH5w) | (z1 & (kClmulH5w << 1)) | (z2 & (kClmulH5w << 2)) | (z3 & (kClmulH5w << 3)) |
                 (z4 & (kClmulH5w << 4));
    if (top) {
        r ^= static_cast<uint64_t>(x) << 31;
    }
    return r;
}

// 32 x 32 -> 64 carry-less product, y given as its 4 holed parts.
CONFKV_CLMUL_FN uint64_t clmul32(uint32_t x, const uint32_t y[4])
{
    const uint64_t x0 = x & kClmulHole, x1 = x & (kClmulHole << 1);
    const uint64_t x2 = x & (kClmulHole << 2), x3 = x & (kClmulHole << 3);
    const uint64_t y0 = y[0], y1 = y[1], y2 = y[2], y3 = y[3];
    const uint64_t z0 = (x0 * y0) ^ (x1 * y3) ^ (x2 * y2) ^ (x3 * y1);
    const uint64_t z1 = (x0 * y1) ^ (x1 * y0) ^ (x2 * y3) ^ (x3 * y2);
    const uint64_t z2 = (x0 * y2) ^ (x1 * y1) ^ (x2 * y0) ^ (x3 * y3);
    const uint64_t z3 = (x0 * y3) ^ (x1 * y2) ^ (x2 * y1) ^ (x3 * y0);
    constexpr uint64_t kH = 0x1111111111111111ull;
    // the four masked residues have no bit in common: adding them is their OR
    return ((z0 & kH) + (z1 & (kH << 1))) + ((z2 & (kH << 2)) + (z3 & (kH << 3)));
}

// The 32 x 32 product of Karatsuba operand k of M: spacing-5 holes when H5.
template <bool H5>
CONFKV_CLMUL_FN uint64_t clmul32_op(uint32_t x, const ClmulConst& c, int k)
{
    if constexpr (H5) {
        return clmul32_h5(x, c.y5[k], ((c.top5 >> k) & 1u) != 0u);
    } else {
        return clmul32(x, c.y[k]);
    }
}

// (ah:al) x M's Karatsuba operands k0 (low word), k0 + 1 (high word), k0 + 2
// (their xor) -> 128 bits, out[0] least significant.
template <bool H5>
CONFKV_CLMUL_FN void clmul64(uint32_t al, uint32_t ah, const ClmulConst& c, int k0, uint32_t out[4])
{
    const uint64_t lo = clmul32_op<H5>(al, c, k0);
    const uint64_t hi = clmul32_op<H5>(ah, c, k0 + 1);
    const uint64_t mid = clmul32_op<H5>(al ^ ah, c, k0 + 2) ^ lo ^ hi;
    out[0] = static_cast<uint32_t>(lo);
    out[1] = static_cast<uint32_t>(lo >> 32) ^ static_cast<uint32_t>(mid);
    out[2] = static_cast<uint32_t>(hi) ^ static_cast<uint32_t>(mid >> 32);
    out[3] = static_cast<uint32_t>(hi >> 32);
}

// x (integer words, x[0] least significant) times M, reduced; x and the
// result in the integer domain. H5 selects the spacing-5 32 x 32 products.
template <bool H5 = false>
CONFKV_CLMUL_FN void clmul_mul_int(const uint32_t x[4], const ClmulConst& c, uint32_t out[4])
{
    uint32_t lo[4], hi[4], s[4];
    clmul64<H5>(x[0], x[1], c, 0, lo);
    clmul64<H5>(x[2], x[3], c, 3, hi);
    clmul64<H5>(x[0] ^ x[2], x[1] ^ x[3], c, 6, s);
    // p = hi << 128 ^ (s ^ lo ^ hi) << 64 ^ lo
    const uint32_t r[8] = {lo[0], lo[1], lo[2] ^ s[0] ^ lo[0] ^ hi[0], lo[3] ^ s[1] ^ lo[1] ^ hi[1],
                           hi[0] ^ s[2] ^ lo[2] ^ hi[2], hi[1] ^ s[3] ^ lo[3] ^ hi[3], hi[2], hi[3]};
    // g = h ^ t, t = (h << 127) ^ (h << 126) ^ (h << 121): only the top word
    uint32_t g[4] = {r[0], r[1], r[2], r[3] ^ (r[0] << 31) ^ (r[0] << 30) ^ (r[0] << 25)};
    for (int w = 0; w < 3; ++w) {
        out[w] = r[4 + w] ^ g[w] ^ ((g[w] >> 1) | (g[w + 1] << 31)) ^ ((g[w] >> 2) | (g[w + 1] << 30)) ^
                 ((g[w] >> 7) | (g[w + 1] << 25));
    }
    out[3] = r[7] ^ g[3] ^ (g[3] >> 1) ^ (g[3] >> 2) ^ (g[3] >> 7);
}

// Raw block words <-> integer words.
CONFKV_CLMUL_FN void clmul_from_raw(const uint32_t raw[4], uint32_t x[4])
{
    for (int w = 0; w < 4; ++w) {
        x[w] = clmul_bswap(raw[3 - w]);
    }
}

CONFKV_CLMUL_FN void clmul_to_raw(const uint32_t x[4], uint32_t raw[4])
{
    for (int w = 0; w < 4; ++w) {
        raw[3 - w] = clmul_bswap(x[w]);
    }
}

// One GHASH Horner step in the integer domain: x <- x * M ^ c (c in integer words).
template <bool H5 = false>
CONFKV_CLMUL_FN void clmul_horner(uint32_t x[4], const ClmulConst& m, const uint32_t c[4])
{
    uint32_t t[4];
    clmul_mul_int<H5>(x, m, t);
    for (int w = 0; w < 4; ++w) {
        x[w] = t[w] ^ c[w];
    }
}

}  // namespace confkv
