/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's AES-128-GCM seal/open path, used by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker. The product (confkv_b200) never links, loads or calls this file.
 *
 * What it restates (reference paths relative to the ConfKV project):
 *   - frame [version=1 | 12-byte IV | ciphertext | 16-byte tag]:
 *       experiments/gpu_kv_seal/gpu/gpu_aesgcm.cu:14-20,
 *       experiments/gpu_kv_seal/native/cpu_seal_openssl.cpp:12-16,133-144
 *   - AES-128 key schedule and block cipher (FIPS-197), as the reference's
 *       expand_aes128_key / aes128_encrypt_block (gpu_aesgcm.cu:304-518).
 *       The S-box is generated from the GF(2^8) inverse and the FIPS-197
 *       affine map rather than stored as a table.
 *   - counter blocks: J0 = IV || 0^31 || 1, data counters start at inc32(J0)
 *       (gpu_aesgcm.cu:586-616,684-692)
 *   - GHASH in the SP 800-38D right-shift form, R = 0xE1 || 0^120
 *       (gpu_aesgcm.cu:195-248), with empty AAD and the final length block
 *       [0^64 || 8*P] (gpu_aesgcm.cu:724-746)
 *   - tag = E_K(J0) xor GHASH (gpu_aesgcm.cu:911-960)
 *   - open: constant-time 16-byte compare plus version == 1, tag read at
 *       13 + P so padded frames are accepted, dst zero-filled on failure
 *       (gpu_aesgcm.cu:964-1034,1650-1660,653-675)
 */
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define ORACLE_VERSION_LEN 1u
#define ORACLE_IV_LEN 12u
#define ORACLE_TAG_LEN 16u
#define ORACLE_HEADER_LEN (ORACLE_VERSION_LEN + ORACLE_IV_LEN)
#define ORACLE_FRAME_OVERHEAD (ORACLE_HEADER_LEN + ORACLE_TAG_LEN)

static uint8_t g_sbox[256];

static uint8_t gf8_mul(uint8_t a, uint8_t b)
{
    uint8_t p = 0;
    for (int i = 0; i < 8; ++i) {
        if (b & 1u) {
            p ^= a;
        }
        const uint8_t hi = (uint8_t)(a & 0x80u);
        a = (uint8_t)(a << 1);
        if (hi) {
            a ^= 0x1bu;
        }
        b >>= 1;
    }
    return p;
}

static uint8_t rotl8(uint8_t x, int s)
{
    return (uint8_t)((x << s) | (x >> (8 - s)));
}

/* FIPS-197 5.1.1: S(x) = affine(x^-1), with 0 mapped through affine(0). */
__attribute__((constructor)) static void oracle_build_sbox(void)
{
    for (int x = 0; x < 256; ++x) {
        uint8_t inv = 0;
        if (x != 0) {
            /* x^254 = x^-1 in GF(2^8) */
            uint8_t acc = 1;
            uint8_t base = (uint8_t)x;
            int e = 254;
            while (e) {
                if (e & 1) {
                    acc = gf8_mul(acc, base);
                }
                base = gf8_mul(base, base);
                e >>= 1;
            }
            inv = acc;
        }
        g_sbox[x] = (uint8_t)(inv ^ rotl8(inv, 1) ^ rotl8(inv, 2) ^
                              rotl8(inv, 3) ^ rotl8(inv, 4) ^ 0x63u);
    }
}

uint8_t oracle_sbox(uint8_t x)
{
    return g_sbox[x];
}

/* FIPS-197 5.2 key expansion, 176 bytes of round keys. */
void oracle_aes128_expand(const uint8_t key[16], uint8_t rk[176])
{
    memcpy(rk, key, 16);
    uint8_t rcon = 1;
    for (int i = 4; i < 44; ++i) {
        uint8_t t[4];
        memcpy(t, rk + 4 * (i - 1), 4);
        if (i % 4 == 0) {
            const uint8_t t0 = t[0];
            t[0] = (uint8_t)(g_sbox[t[1]] ^ rcon);
            t[1] = g_sbox[t[2]];
            t[2] = g_sbox[t[3]];
            t[3] = g_sbox[t0];
            rcon = gf8_mul(rcon, 2);
        }
        for (int j = 0; j < 4; ++j) {
            rk[4 * i + j] = (uint8_t)(rk[4 * (i - 4) + j] ^ t[j]);
        }
    }
}

/* FIPS-197 5.1 cipher; state byte s[r + 4c] is row r, column c. */
void oracle_aes128_encrypt_rk(const uint8_t rk[176], const uint8_t in[16], uint8_t out[16])
{
    uint8_t s[16];
    for (int i = 0; i < 16; ++i) {
        s[i] = (uint8_t)(in[i] ^ rk[i]);
    }
    for (int round = 1; round <= 10; ++round) {
        uint8_t t[16];
        /* SubBytes + ShiftRows: row r rotates left by r columns */
        for (int c = 0; c < 4; ++c) {
            for (int r = 0; r < 4; ++r) {
                t[r + 4 * c] = g_sbox[s[r + 4 * ((c + r) & 3)]];
            }
        }
        if (round != 10) {
            for (int c = 0; c < 4; ++c) {
                const uint8_t a0 = t[4 * c], a1 = t[4 * c + 1];
                const uint8_t a2 = t[4 * c + 2], a3 = t[4 * c + 3];
                t[4 * c + 0] = (uint8_t)(gf8_mul(a0, 2) ^ gf8_mul(a1, 3) ^ a2 ^ a3);
                t[4 * c + 1] = (uint8_t)(a0 ^ gf8_mul(a1, 2) ^ gf8_mul(a2, 3) ^ a3);
                t[4 * c + 2] = (uint8_t)(a0 ^ a1 ^ gf8_mul(a2, 2) ^ gf8_mul(a3, 3));
                t[4 * c + 3] = (uint8_t)(gf8_mul(a0, 3) ^ a1 ^ a2 ^ gf8_mul(a3, 2));
            }
        }
        for (int i = 0; i < 16; ++i) {
            s[i] = (uint8_t)(t[i] ^ rk[16 * round + i]);
        }
    }
    memcpy(out, s, 16);
}

void oracle_aes128_encrypt(const uint8_t key[16], const uint8_t in[16], uint8_t out[16])
{
    uint8_t rk[176];
    oracle_aes128_expand(key, rk);
    oracle_aes128_encrypt_rk(rk, in, out);
}

/* ---- GF(2^128), SP 800-38D bit order: bit 0 is the MSB of byte 0. ---- */

typedef struct {
    uint64_t hi; /* bytes 0..7, big-endian */
    uint64_t lo; /* bytes 8..15, big-endian */
} oracle_u128;

static oracle_u128 load_be(const uint8_t p[16])
{
    oracle_u128 x = {0, 0};
    for (int i = 0; i < 8; ++i) {
        x.hi = (x.hi << 8) | p[i];
        x.lo = (x.lo << 8) | p[8 + i];
    }
    return x;
}

static void store_be(uint8_t p[16], oracle_u128 x)
{
    for (int i = 7; i >= 0; --i) {
        p[i] = (uint8_t)x.hi;
        p[8 + i] = (uint8_t)x.lo;
        x.hi >>= 8;
        x.lo >>= 8;
    }
}

/* SP 800-38D Algorithm 1 (right-shift multiply). */
static oracle_u128 gf128_mul(oracle_u128 x, oracle_u128 y)
{
    oracle_u128 z = {0, 0};
    oracle_u128 v = y;
    for (int i = 0; i < 128; ++i) {
        const uint64_t bit = i < 64 ? (x.hi >> (63 - i)) & 1u : (x.lo >> (127 - i)) & 1u;
        const uint64_t m = 0 - bit;
        z.hi ^= v.hi & m;
        z.lo ^= v.lo & m;
        const uint64_t lsb = v.lo & 1u;
        v.lo = (v.lo >> 1) | (v.hi << 63);
        v.hi = (v.hi >> 1) ^ (0xe100000000000000ull & (0 - lsb));
    }
    return z;
}

/* Byte-level GF(2^128) multiply, exported for host-logic checks. */
void oracle_gf128_mul(const uint8_t a[16], const uint8_t b[16], uint8_t out[16])
{
    store_be(out, gf128_mul(load_be(a), load_be(b)));
}

/*
 * GHASH_H over `len` bytes of data (zero-padded to a block) followed by the
 * length block [0^64 || 8*len]: exactly the hash the reference computes over
 * the ciphertext with empty AAD.
 */
void oracle_ghash_ct(const uint8_t h_bytes[16], const uint8_t* data, size_t len, uint8_t out[16])
{
    const oracle_u128 h = load_be(h_bytes);
    oracle_u128 y = {0, 0};
    size_t off = 0;
    while (off < len) {
        uint8_t blk[16] = {0};
        const size_t n = len - off < 16 ? len - off : 16;
        memcpy(blk, data + off, n);
        const oracle_u128 x = load_be(blk);
        y.hi ^= x.hi;
        y.lo ^= x.lo;
        y = gf128_mul(y, h);
        off += n;
    }
    y.lo ^= (uint64_t)len * 8u;
    y = gf128_mul(y, h);
    store_be(out, y);
}

static void counter_block(const uint8_t iv[12], uint32_t ctr, uint8_t blk[16])
{
    memcpy(blk, iv, 12);
    blk[12] = (uint8_t)(ctr >> 24);
    blk[13] = (uint8_t)(ctr >> 16);
    blk[14] = (uint8_t)(ctr >> 8);
    blk[15] = (uint8_t)ctr;
}

static void ctr_xor(const uint8_t rk[176], const uint8_t iv[12], const uint8_t* in,
                    uint8_t* out, size_t len)
{
    uint32_t ctr = 2; /* inc32(J0) */
    for (size_t off = 0; off < len; off += 16, ++ctr) {
        uint8_t cb[16], ks[16];
        counter_block(iv, ctr, cb);
        oracle_aes128_encrypt_rk(rk, cb, ks);
        const size_t n = len - off < 16 ? len - off : 16;
        for (size_t j = 0; j < n; ++j) {
            out[off + j] = (uint8_t)(in[off + j] ^ ks[j]);
        }
    }
}

static void compute_tag(const uint8_t rk[176], const uint8_t iv[12], const uint8_t* ct,
                        size_t len, uint8_t tag[16])
{
    uint8_t zero[16] = {0}, h[16], j0[16], ej0[16], s[16];
    oracle_aes128_encrypt_rk(rk, zero, h);
    oracle_ghash_ct(h, ct, len, s);
    counter_block(iv, 1, j0);
    oracle_aes128_encrypt_rk(rk, j0, ej0);
    for (int i = 0; i < 16; ++i) {
        tag[i] = (uint8_t)(ej0[i] ^ s[i]);
    }
}

size_t oracle_frame_size(size_t plaintext_len)
{
    return plaintext_len + ORACLE_FRAME_OVERHEAD;
}

/*
 * Seal with a caller-chosen IV into [1 | iv | C | T].
 * Returns 0 on success, -1 on a bad argument (null pointer or short dst),
 * -2 if the plaintext needs more than 2^32 - 2 counter blocks.
 */
int oracle_gcm_seal(const uint8_t key[16], const uint8_t iv[12], const uint8_t* src,
                    size_t len, uint8_t* frame, size_t frame_cap)
{
    if (key == NULL || iv == NULL || frame == NULL || (src == NULL && len != 0)) {
        return -1;
    }
    if (frame_cap < oracle_frame_size(len)) {
        return -1;
    }
    if ((len + 15u) / 16u > 0xfffffffeull) {
        return -2;
    }
    uint8_t rk[176];
    oracle_aes128_expand(key, rk);
    frame[0] = 1;
    memcpy(frame + 1, iv, 12);
    ctr_xor(rk, iv, src, frame + ORACLE_HEADER_LEN, len);
    compute_tag(rk, iv, frame + ORACLE_HEADER_LEN, len, frame + ORACLE_HEADER_LEN + len);
    return 0;
}

/*
 * Authentication-gated open of a frame holding `plaintext_len` bytes of
 * ciphertext (frame_len may be larger: padded frames are accepted and the tag
 * is read at 13 + plaintext_len). Returns 1 if the tag and version match and
 * dst holds the plaintext, 0 if authentication failed and dst was zero-filled,
 * -1 on a bad argument.
 */
int oracle_gcm_open(const uint8_t key[16], const uint8_t* frame, size_t frame_len,
                    uint8_t* dst, size_t plaintext_len)
{
    if (key == NULL || frame == NULL || (dst == NULL && plaintext_len != 0)) {
        return -1;
    }
    if (frame_len < oracle_frame_size(plaintext_len)) {
        return -1;
    }
    uint8_t rk[176], tag[16];
    oracle_aes128_expand(key, rk);
    const uint8_t* iv = frame + 1;
    const uint8_t* ct = frame + ORACLE_HEADER_LEN;
    compute_tag(rk, iv, ct, plaintext_len, tag);
    unsigned diff = 0;
    for (int i = 0; i < 16; ++i) {
        diff |= (unsigned)(tag[i] ^ ct[plaintext_len + i]);
    }
    const int ok = (frame[0] == 1) && diff == 0;
    if (!ok) {
        if (plaintext_len) {
            memset(dst, 0, plaintext_len);
        }
        return 0;
    }
    ctr_xor(rk, iv, ct, dst, plaintext_len);
    return 1;
}
