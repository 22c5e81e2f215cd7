// Host-side AES-128 / GHASH helpers used once per key at key_create time:
// the S-box and T-tables, the key schedule, H = E_K(0), and the 4-bit GHASH
// multiplication tables the kernels read. No CUDA in here.
#pragma once

#include <cstddef>
#include <cstdint>

#include "gh5.cuh"

namespace confkv {

// GF(2^128) element in the SP 800-38D convention: hi holds bytes 0..7 of the
// block big-endian, lo bytes 8..15; bit 0 of the block (MSB of byte 0) is the
// coefficient of x^0.
struct Gf128 {
    uint64_t hi;
    uint64_t lo;
};

constexpr int kAesRounds = 10;
constexpr int kRoundKeyWords = 4 * (kAesRounds + 1);  // 44

// 4-bit GHASH table: 32 nibble positions x 16 values x 16 bytes = 8 KiB.
// Position p = 2*j + h covers byte j of the block, h = 0 for its low nibble
// and h = 1 for its high nibble. Entry [p][v] holds the raw 16 block bytes of
// (block whose byte j is v << (4*h)) * M.
constexpr int kGhashPositions = 32;
constexpr int kGhashTableBytes = kGhashPositions * 16 * 16;

// Number of precomputed H^(2^k) tables kept per key (exponents < 2^36).
constexpr int kPow2Tables = 36;

const uint8_t* aes_sbox();

// T0[x] as a little-endian word holding bytes (2*S[x], S[x], S[x], 3*S[x]).
// T1..T3 are T0 rotated left by 8, 16 and 24 bits.
void aes_t_tables(uint32_t t[4][256]);

// FIPS-197 key expansion; round key r word c is the little-endian load of
// bytes 16*r + 4*c .. 16*r + 4*c + 3.
void aes128_expand_le(const uint8_t key[16], uint32_t rk[kRoundKeyWords]);

void aes128_encrypt_block(const uint32_t rk[kRoundKeyWords], const uint8_t in[16],
                          uint8_t out[16]);

Gf128 gf_load(const uint8_t b[16]);
void gf_store(uint8_t b[16], Gf128 x);
Gf128 gf_mul(Gf128 a, Gf128 b);
Gf128 gf_mul_x(Gf128 v);
Gf128 gf_pow(Gf128 h, uint64_t e);

// Fill `out` (kGhashTableBytes) with the 4-bit table for multiplier m.
void ghash_table(Gf128 m, uint8_t* out);

// Fill `out` (kGh5CompactBytes, gh5.cuh) with the kGhW-bit-window table for
// m: entry (g, v) at (g * kGh5Values + v) * 16.
void ghash_table5(Gf128 m, uint8_t* out);

}  // namespace confkv
