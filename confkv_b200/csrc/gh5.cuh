// GHASH multiplication by a fixed M with 5-bit windows: the 128 bits of a
// block, read in raw order (raw bit r = bit r % 32 of little-endian word
// r / 32), are cut into 26 groups of 5 consecutive raw bits (the last has 3).
// Entry (g, v) of M's table is the sum over the set bits b of v of
// x^e(5g + b) M, e(r) being the SP 800-38D index of raw bit r (byte
// 4 (r / 32) + (r % 32) / 8, bit 7 - r % 8 counted from the byte's MSB), so
// x M = XOR over g of entry (g, field g of x): 26 lookups of 16 B instead of
// the 32 of 4-bit tables. Each group's field is one contiguous run of a word
// (or of two adjacent words), so its shared-memory address takes one shift
// and one LOP3. Host and device share the field extraction.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define CONFKV_GH5_FN __host__ __device__ __forceinline__
#else
#define CONFKV_GH5_FN inline
#endif

namespace confkv {

constexpr int kGh5Groups = 26;
constexpr int kGh5Values = 32;
constexpr int kGh5CompactBytes = kGh5Groups * kGh5Values * 16;  // 13,312 B
// Replicated shared-memory layout: row (g, v) = 8 replicas of the entry
// (128 B, one bank sweep) at g * 4096 + v * 128; lane l reads replica l & 7,
// so the 8 lanes of an LDS.128 phase hit 8 distinct bank groups whatever v.
constexpr int kGh5GroupStride = kGh5Values * 128;
constexpr int kGh5RepBytes = kGh5Groups * kGh5GroupStride;     // 106,496 B

// SP 800-38D bit index (x^e) of raw bit r.
CONFKV_GH5_FN int gh5_gcm_index(int r)
{
    const int w = r >> 5, q = r & 31;
    return 8 * (4 * w + (q >> 3)) + (7 - (q & 7));
}

// Field g of x (raw words), shifted to bits 7..11 with the other bits of the
// result below bit 7 or above bit 11 left as they come: the caller masks
// with 0xF80. Group g starts at raw bit 5g = bit s of word w.
template <int G>
CONFKV_GH5_FN uint32_t gh5_field_at7(const uint32_t x[4])
{
    constexpr int r0 = 5 * G;
    constexpr int w = r0 >> 5;
    constexpr int s = r0 & 31;
    if constexpr (s < 7) {
        return x[w] << (7 - s);
    } else if constexpr (s + 5 <= 32 || w == 3) {
        return x[w] >> (s - 7);
    } else {
        // bits s..31 of word w, then bits 0.. of word w + 1
        return (x[w] >> (s - 7)) | (x[w + 1] << (32 - (s - 7)));
    }
}

}  // namespace confkv
