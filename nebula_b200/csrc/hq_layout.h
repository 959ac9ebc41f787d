// hq_layout.h -- the tile order of packed weights (host and device).
//
// A strip s is 16 output columns [16s, 16s+16); a strip group sg = s/8 is 128
// columns (the last group may hold fewer strips); a k-block kb is 64 k.
// A chunk (s, kb) = 16 columns x 64 k, kChunkBytes(wbits) bytes, stored at
//     (sg*8*KB + kb*width(sg) + s%8) * chunk_bytes          (KB = K/64)
// so the chunks of one strip group are one contiguous run along k, and a run of
// consecutive "units" (sg, kb) -- one k-block of one strip group -- is one
// contiguous byte span for any unit range: a single bulk copy moves it.
//
// Inside a chunk, lane l = 4g + t (g = 0..7, t = 0..3) of a warp owns
// chunk_bytes/32 bytes at l*chunk_bytes/32, as little-endian 32-bit words:
//   int4:    word j (0..3) = column 16s + g + 8*(j>>1), k = 64kb + 16t + 8*(j&1) + e,
//            e = 0..7, 4-bit code u = q + 8 at nibble u4_pos(e):
//            e 0 1 2 3 4 5 6 7 -> nibble 0 4 2 6 1 5 3 7;
//   ternary: word j (0..1) = column 16s + g + 8*j, k = 64kb + 16t + e, e = 0..15,
//            2-bit code c = q + 1 at field (e>>1) + 8*(e&1).
// A lane's words therefore hold exactly the A-fragment elements of
// mma.m16n8k16 for rows g and g+8 once the k index inside each 16-wide MMA
// step is relabelled (the relabelling is applied identically to the
// activation fragment, so the dot product is unchanged), and each word is 8
// (int4) or 16 (ternary) consecutive k of one column, which is what the
// tensor-core prefill kernel stores as one 16-byte K-major smem vector.
// In an int4 word the codes of k-pairs (e0,e1) and (e2,e3) sit in the low
// nibble of each byte (nibbles 0/4 and 2/6) and (e4,e5), (e6,e7) in the high
// nibble (1/5 and 3/7): one MMA step draws all its pairs from one of the two
// nibble classes, so a class is expanded with a single mask per pair.
//
// TILE_U4_K32, the layout for scale groups of 32 k: the same chunks, words and
// nibble order, but word j of lane t holds k = 64kb + 8t + 32*(j&1) + e.  The
// MMA steps built from word j = 0 (steps 0, 1) then lie in k [0, 32) of the
// block and those from j = 1 (steps 2, 3) in [32, 64): each step belongs to
// one scale group.  The activation fragments relabel k the same way.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define HQ_HD __host__ __device__ __forceinline__
#else
#define HQ_HD inline
#endif

namespace hq {

constexpr int kStripCols = 16;
constexpr int kGroupStrips = 8;
constexpr int kGroupCols = kStripCols * kGroupStrips;  // 128
constexpr int kBlockK = 64;

HQ_HD int chunk_bytes(int wbits) { return wbits == 4 ? 512 : 256; }

struct TileGeom {
    int K, N, wbits;
    int KB;   // k-blocks
    int NS;   // strips
    int NSG;  // strip groups
    int CB;   // chunk bytes

    HQ_HD TileGeom(int K_, int N_, int wbits_)
        : K(K_), N(N_), wbits(wbits_), KB(K_ / kBlockK), NS(N_ / kStripCols),
          NSG((N_ / kStripCols + kGroupStrips - 1) / kGroupStrips), CB(chunk_bytes(wbits_)) {}

    HQ_HD int width(int sg) const {
        int w = NS - kGroupStrips * sg;
        return w < kGroupStrips ? w : kGroupStrips;
    }
    // Units are (sg, kb) pairs in sg-major order.
    HQ_HD long long units() const { return (long long)NSG * KB; }
    // Byte offset of the start of unit u; u == units() gives the end of the
    // tensor (the last strip group may be narrower than 8 strips, so the end is
    // not where a full group would end).
    HQ_HD size_t unit_offset(long long u) const {
        if (u >= units()) return bytes();
        long long sg = u / KB, kb = u % KB;
        return ((size_t)sg * kGroupStrips * KB + (size_t)kb * width((int)sg)) * (size_t)CB;
    }
    HQ_HD size_t chunk_offset(int s, int kb) const {
        int sg = s / kGroupStrips;
        return ((size_t)sg * kGroupStrips * KB + (size_t)kb * width(sg) + (size_t)(s % kGroupStrips)) * (size_t)CB;
    }
    HQ_HD size_t bytes() const { return (size_t)KB * NS * CB; }
};

// Position (nibble or 2-bit field index) of in-word element e.
HQ_HD int u4_pos(int e) { return 2 * ((e >> 1) & 1) + ((e >> 2) & 1) + 4 * (e & 1); }
HQ_HD int t2_pos(int e) { return (e >> 1) + 8 * (e & 1); }

// Reorder the 8 nibbles of a linear word (k-offset e at nibble e) into tile order.
HQ_HD uint32_t u4_linear_to_tile(uint32_t w) {
    uint32_t o = 0;
    for (int e = 0; e < 8; ++e) o |= ((w >> (4 * e)) & 0xFu) << (4 * u4_pos(e));
    return o;
}
HQ_HD uint32_t u4_tile_to_linear(uint32_t w) {
    uint32_t o = 0;
    for (int e = 0; e < 8; ++e) o |= ((w >> (4 * u4_pos(e))) & 0xFu) << (4 * e);
    return o;
}
HQ_HD uint32_t t2_linear_to_tile(uint32_t w) {
    uint32_t o = 0;
    for (int e = 0; e < 16; ++e) o |= ((w >> (2 * e)) & 0x3u) << (2 * t2_pos(e));
    return o;
}
HQ_HD uint32_t t2_tile_to_linear(uint32_t w) {
    uint32_t o = 0;
    for (int e = 0; e < 16; ++e) o |= ((w >> (2 * t2_pos(e))) & 0x3u) << (2 * e);
    return o;
}

// For tile word (s, kb, lane, j): the output column and the linear-format
// word row (kw) it mirrors.  int4 linear words hold 8 k (kw = k/8), ternary
// linear words hold 16 k (kw = k/16).  k32: the TILE_U4_K32 order.
HQ_HD void tile_word_source(int wbits, int s, int kb, int lane, int j, int* col, int* kw, bool k32 = false) {
    int g = lane >> 2, t = lane & 3;
    if (wbits == 4) {
        *col = s * kStripCols + g + 8 * (j >> 1);
        *kw = k32 ? (kb * kBlockK + 8 * t + 32 * (j & 1)) / 8 : (kb * kBlockK + 16 * t + 8 * (j & 1)) / 8;
    } else {
        *col = s * kStripCols + g + 8 * j;
        *kw = (kb * kBlockK + 16 * t) / 16;
    }
}

}  // namespace hq
