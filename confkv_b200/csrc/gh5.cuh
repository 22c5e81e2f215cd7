// GHASH multiplication by a fixed M with W-bit windows (W = kGhW, 5 or 6):
// the 128 bits of a block, read in raw order (raw bit r = bit r % 32 of
// little-endian word r / 32), are cut into ceil(128 / W) groups of W
// consecutive raw bits (the last one shorter). Entry (g, v) of M's table is
// the sum over the set bits b of v of x^e(W g + b) M, e(r) being the
// SP 800-38D index of raw bit r (byte 4 (r / 32) + (r % 32) / 8, bit
// 7 - r % 8 counted from the byte's MSB), so x M = XOR over g of entry
// (g, field g of x): 26 (W = 5) or 22 (W = 6) lookups of 16 B instead of the
// 32 of 4-bit tables. Each group's field is one contiguous run of a word (or
// of two adjacent words), so its shared-memory address takes one shift and
// one LOP3. Host and device share the field extraction.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define CONFKV_GH5_FN __host__ __device__ __forceinline__
#else
#define CONFKV_GH5_FN inline
#endif

namespace confkv {

// Window width of the batched GHASH passes' tables: 5 or 6 bits (6: 22
// lookups per multiply; the host tests build both).
#ifndef CONFKV_GH_WINDOW
#define CONFKV_GH_WINDOW 6
#endif
constexpr int kGhW = CONFKV_GH_WINDOW;
static_assert(kGhW == 5 || kGhW == 6, "window tables are 5 or 6 bits wide");
constexpr int kGh5Groups = (128 + kGhW - 1) / kGhW;
constexpr int kGh5Values = 1 << kGhW;
constexpr int kGh5CompactBytes = kGh5Groups * kGh5Values * 16;
// Replicated shared-memory layout: row (g, v) = 8 replicas of the entry
// (128 B, one bank sweep) at g * (values * 128) + v * 128; lane l reads
// replica l & 7, so the 8 lanes of an LDS.128 phase hit 8 distinct bank
// groups whatever v.
constexpr int kGh5GroupStride = kGh5Values * 128;
constexpr int kGh5RepBytes = kGh5Groups * kGh5GroupStride;
constexpr uint32_t kGh5Mask7 = static_cast<uint32_t>(kGh5Values - 1) << 7;  // the field at bits 7 ..

// SP 800-38D bit index (x^e) of raw bit r.
CONFKV_GH5_FN int gh5_gcm_index(int r)
{
    const int w = r >> 5, q = r & 31;
    return 8 * (4 * w + (q >> 3)) + (7 - (q & 7));
}

// Field g of x (raw words), shifted to start at bit 7, with the other bits
// of the result left as they come: the caller masks with kGh5Mask7. Group g
// starts at raw bit kGhW g = bit s of word w.
template <int G>
CONFKV_GH5_FN uint32_t gh5_field_at7(const uint32_t x[4])
{
    constexpr int r0 = kGhW * G;
    constexpr int w = r0 >> 5;
    constexpr int s = r0 & 31;
    if constexpr (s < 7) {
        return x[w] << (7 - s);
    } else if constexpr (s + kGhW <= 32 || w == 3) {
        return x[w] >> (s - 7);
    } else {
        // bits s..31 of word w, then bits 0.. of word w + 1
        return (x[w] >> (s - 7)) | (x[w + 1] << (32 - (s - 7)));
    }
}

}  // namespace confkv
