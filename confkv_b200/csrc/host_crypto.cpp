// Host-side AES-128 / GHASH helpers. See host_crypto.h.
//
// The AES S-box is derived from its definition (FIPS-197 5.1.1: multiplicative
// inverse in GF(2^8) followed by the affine map) rather than stored. GHASH
// arithmetic follows NIST SP 800-38D (right-shift multiply, R = 0xE1 || 0^120),
// the same field convention as the reference's gf_mul
// (experiments/gpu_kv_seal/gpu/gpu_aesgcm.cu:195-248).
#include "host_crypto.h"

#include <cstring>

namespace confkv {
namespace {

uint8_t gf8_mul(uint8_t a, uint8_t b)
{
    uint8_t p = 0;
    while (b) {
        if (b & 1u) {
            p ^= a;
        }
        a = static_cast<uint8_t>((a << 1) ^ ((a & 0x80u) ? 0x1bu : 0u));
        b >>= 1;
    }
    return p;
}

uint8_t rotl8(uint8_t x, int s)
{
    return static_cast<uint8_t>((x << s) | (x >> (8 - s)));
}

struct SboxHolder {
    uint8_t s[256];
    SboxHolder()
    {
        for (int x = 0; x < 256; ++x) {
            uint8_t inv = 0;
            if (x) {
                // x^254 = x^-1
                uint8_t acc = 1, base = static_cast<uint8_t>(x);
                for (int e = 254; e; e >>= 1) {
                    if (e & 1) {
                        acc = gf8_mul(acc, base);
                    }
                    base = gf8_mul(base, base);
                }
                inv = acc;
            }
            s[x] = static_cast<uint8_t>(inv ^ rotl8(inv, 1) ^ rotl8(inv, 2) ^ rotl8(inv, 3) ^
                                        rotl8(inv, 4) ^ 0x63u);
        }
    }
};

const SboxHolder& sbox_holder()
{
    static const SboxHolder h;
    return h;
}

uint32_t le32(const uint8_t* p)
{
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
           (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
}

uint32_t rotl32(uint32_t x, int s)
{
    return (x << s) | (x >> (32 - s));
}

}  // namespace

const uint8_t* aes_sbox()
{
    return sbox_holder().s;
}

void aes_t_tables(uint32_t t[4][256])
{
    const uint8_t* s = aes_sbox();
    for (int x = 0; x < 256; ++x) {
        const uint8_t a = s[x];
        const uint8_t a2 = gf8_mul(a, 2);
        const uint8_t a3 = static_cast<uint8_t>(a2 ^ a);
        const uint32_t w = static_cast<uint32_t>(a2) | (static_cast<uint32_t>(a) << 8) |
                           (static_cast<uint32_t>(a) << 16) | (static_cast<uint32_t>(a3) << 24);
        t[0][x] = w;
        t[1][x] = rotl32(w, 8);
        t[2][x] = rotl32(w, 16);
        t[3][x] = rotl32(w, 24);
    }
}

void aes128_expand_le(const uint8_t key[16], uint32_t rk[kRoundKeyWords])
{
    const uint8_t* s = aes_sbox();
    uint8_t w[4 * kRoundKeyWords];
    std::memcpy(w, key, 16);
    uint8_t rcon = 1;
    for (int i = 4; i < kRoundKeyWords; ++i) {
        uint8_t t[4];
        std::memcpy(t, w + 4 * (i - 1), 4);
        if (i % 4 == 0) {
            const uint8_t t0 = t[0];
            t[0] = static_cast<uint8_t>(s[t[1]] ^ rcon);
            t[1] = s[t[2]];
            t[2] = s[t[3]];
            t[3] = s[t0];
            rcon = gf8_mul(rcon, 2);
        }
        for (int j = 0; j < 4; ++j) {
            w[4 * i + j] = static_cast<uint8_t>(w[4 * (i - 4) + j] ^ t[j]);
        }
    }
    for (int i = 0; i < kRoundKeyWords; ++i) {
        rk[i] = le32(w + 4 * i);
    }
}

void aes128_encrypt_block(const uint32_t rk[kRoundKeyWords], const uint8_t in[16],
                          uint8_t out[16])
{
    struct TTables {
        uint32_t t[4][256];
        TTables() { aes_t_tables(t); }
    };
    static const TTables tt;  // thread-safe one-time init
    const auto& t = tt.t;
    const uint8_t* s = aes_sbox();
    uint32_t w[4];
    for (int c = 0; c < 4; ++c) {
        w[c] = le32(in + 4 * c) ^ rk[c];
    }
    for (int r = 1; r < kAesRounds; ++r) {
        uint32_t n[4];
        for (int c = 0; c < 4; ++c) {
            n[c] = t[0][w[c] & 0xff] ^ t[1][(w[(c + 1) & 3] >> 8) & 0xff] ^
                   t[2][(w[(c + 2) & 3] >> 16) & 0xff] ^ t[3][w[(c + 3) & 3] >> 24] ^
                   rk[4 * r + c];
        }
        std::memcpy(w, n, sizeof(w));
    }
    for (int c = 0; c < 4; ++c) {
        const uint32_t v = static_cast<uint32_t>(s[w[c] & 0xff]) |
                           (static_cast<uint32_t>(s[(w[(c + 1) & 3] >> 8) & 0xff]) << 8) |
                           (static_cast<uint32_t>(s[(w[(c + 2) & 3] >> 16) & 0xff]) << 16) |
                           (static_cast<uint32_t>(s[w[(c + 3) & 3] >> 24]) << 24);
        const uint32_t o = v ^ rk[4 * kAesRounds + c];
        out[4 * c + 0] = static_cast<uint8_t>(o);
        out[4 * c + 1] = static_cast<uint8_t>(o >> 8);
        out[4 * c + 2] = static_cast<uint8_t>(o >> 16);
        out[4 * c + 3] = static_cast<uint8_t>(o >> 24);
    }
}

Gf128 gf_load(const uint8_t b[16])
{
    Gf128 x{0, 0};
    for (int i = 0; i < 8; ++i) {
        x.hi = (x.hi << 8) | b[i];
        x.lo = (x.lo << 8) | b[8 + i];
    }
    return x;
}

void gf_store(uint8_t b[16], Gf128 x)
{
    for (int i = 7; i >= 0; --i) {
        b[i] = static_cast<uint8_t>(x.hi);
        b[8 + i] = static_cast<uint8_t>(x.lo);
        x.hi >>= 8;
        x.lo >>= 8;
    }
}

Gf128 gf_mul_x(Gf128 v)
{
    const uint64_t lsb = v.lo & 1u;
    Gf128 r;
    r.lo = (v.lo >> 1) | (v.hi << 63);
    r.hi = (v.hi >> 1) ^ (0xe100000000000000ull & (0 - lsb));
    return r;
}

Gf128 gf_mul(Gf128 a, Gf128 b)
{
    Gf128 z{0, 0};
    Gf128 v = b;
    for (int i = 0; i < 128; ++i) {
        const uint64_t bit = i < 64 ? (a.hi >> (63 - i)) & 1u : (a.lo >> (127 - i)) & 1u;
        const uint64_t m = 0 - bit;
        z.hi ^= v.hi & m;
        z.lo ^= v.lo & m;
        v = gf_mul_x(v);
    }
    return z;
}

Gf128 gf_pow(Gf128 h, uint64_t e)
{
    Gf128 r{0x8000000000000000ull, 0};  // multiplicative identity x^0
    Gf128 base = h;
    while (e) {
        if (e & 1u) {
            r = gf_mul(r, base);
        }
        base = gf_mul(base, base);
        e >>= 1;
    }
    return r;
}

void ghash_table(Gf128 m, uint8_t* out)
{
    // basis[b] = x^b * m: the product for a block with only bit b set.
    Gf128 basis[128];
    basis[0] = m;
    for (int b = 1; b < 128; ++b) {
        basis[b] = gf_mul_x(basis[b - 1]);
    }
    for (int j = 0; j < 16; ++j) {
        for (int h = 0; h < 2; ++h) {
            const int p = 2 * j + h;
            for (int v = 0; v < 16; ++v) {
                const unsigned byte_val = static_cast<unsigned>(v) << (4 * h);
                Gf128 acc{0, 0};
                for (int k = 0; k < 8; ++k) {
                    if (byte_val & (1u << k)) {
                        // byte value bit k (LSB = 0) is block bit 8*j + 7 - k
                        const Gf128 e = basis[8 * j + 7 - k];
                        acc.hi ^= e.hi;
                        acc.lo ^= e.lo;
                    }
                }
                gf_store(out + (p * 16 + v) * 16, acc);
            }
        }
    }
}

void ghash_table5(Gf128 m, uint8_t* out)
{
    Gf128 basis[128];  // basis[e] = x^e * m
    basis[0] = m;
    for (int b = 1; b < 128; ++b) {
        basis[b] = gf_mul_x(basis[b - 1]);
    }
    for (int g = 0; g < kGh5Groups; ++g) {
        for (int v = 0; v < kGh5Values; ++v) {
            Gf128 acc{0, 0};
            for (int b = 0; b < kGhW; ++b) {
                const int r = kGhW * g + b;
                if (((v >> b) & 1) != 0 && r < 128) {
                    const Gf128 e = basis[gh5_gcm_index(r)];
                    acc.hi ^= e.hi;
                    acc.lo ^= e.lo;
                }
            }
            gf_store(out + (g * kGh5Values + v) * 16, acc);
        }
    }
}

}  // namespace confkv
