// hq_decode_frag.cuh -- register fragments of the mma.sync decode kernel: the
// activation (B) fragments read from the staged activation tiles, and the
// weight (A) fragments expanded from a lane's tile-order words.
#pragma once

#include "hq_common.cuh"
#include "hq_layout.h"

namespace hq {
namespace frag {

// fp16 / bf16 activations: the 16 k (4 MMA steps) of one token row for this lane.
template <typename AT>
struct XFrag {
    uint4 a, b;
    // TMA tile: row `r`, 16-byte chunks c at ((c ^ (r & 7)) << 4) (128B swizzle).
    __device__ __forceinline__ void load(const uint8_t* tile, int r, int t) {
        const uint8_t* row = tile + r * 128;
        a = *reinterpret_cast<const uint4*>(row + (((2 * t) ^ (r & 7)) << 4));
        b = *reinterpret_cast<const uint4*>(row + (((2 * t + 1) ^ (r & 7)) << 4));
    }
    __device__ __forceinline__ uint32_t b0(int step) const {
        return step == 0 ? a.x : step == 1 ? a.z : step == 2 ? b.x : b.z;
    }
    __device__ __forceinline__ uint32_t b1(int step) const {
        return step == 0 ? a.y : step == 1 ? a.w : step == 2 ? b.y : b.w;
    }
};

// fp32 activations (padded rows of kBlockK floats + 16 bytes): x = hi + lo with
// hi = fp16(x), lo = fp16(x - hi); two MMAs per step keep the product accurate
// to ~2^-22 relative.
struct XFragF32 {
    static constexpr int kRowBytes = kBlockK * 4 + 16;
    uint32_t hi[8], lo[8];
    __device__ __forceinline__ void load(const uint8_t* tile, int r, int t) {
        const uint8_t* sp = tile + r * kRowBytes + 16 * t * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 q = *reinterpret_cast<const uint4*>(sp + 16 * i);
            float4 v = make_float4(__uint_as_float(q.x), __uint_as_float(q.y), __uint_as_float(q.z),
                                   __uint_as_float(q.w));
            __half2 h0 = __floats2half2_rn(v.x, v.y);
            __half2 h1 = __floats2half2_rn(v.z, v.w);
            float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
            __half2 l0 = __floats2half2_rn(v.x - f0.x, v.y - f0.y);
            __half2 l1 = __floats2half2_rn(v.z - f1.x, v.w - f1.y);
            hi[2 * i] = *reinterpret_cast<uint32_t*>(&h0);
            hi[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h1);
            lo[2 * i] = *reinterpret_cast<uint32_t*>(&l0);
            lo[2 * i + 1] = *reinterpret_cast<uint32_t*>(&l1);
        }
    }
};

// The MMA input type: bf16 activations compute in bf16, fp16 and fp32 in fp16.
template <typename AT>
struct ComputeType {
    static constexpr bool bf16 = false;
};
template <>
struct ComputeType<__nv_bfloat16> {
    static constexpr bool bf16 = true;
};

// A fragments (4 regs) of each of the four m16n8k16 steps from a lane's chunk
// words: exact q = u - 8 (int4) / t = c - 1 (ternary), or the code u itself
// when kUnsigned (the reference's u * scale + bias form).
template <int WBITS, bool kBF16, bool kUnsigned>
struct WFrag {
    uint32_t r[4][4];  // [step][reg]
    __device__ __forceinline__ void expand(uint32_t w, uint32_t (&o)[4]) {
        if constexpr (kBF16)
            dequant_u4_bf16<kUnsigned>(w, o);
        else
            dequant_u4_f16<kUnsigned>(w, o);
    }
    __device__ __forceinline__ void build(uint4 w) {
        if constexpr (WBITS == 4) {
            uint32_t g0[4], g8[4];
            // words: x = row g k0..7, y = row g k8..15, z = row g+8 k0..7, w = row g+8 k8..15
            expand(w.x, g0);
            expand(w.z, g8);
            r[0][0] = g0[0]; r[0][1] = g8[0]; r[0][2] = g0[1]; r[0][3] = g8[1];
            r[1][0] = g0[2]; r[1][1] = g8[2]; r[1][2] = g0[3]; r[1][3] = g8[3];
            expand(w.y, g0);
            expand(w.w, g8);
            r[2][0] = g0[0]; r[2][1] = g8[0]; r[2][2] = g0[1]; r[2][3] = g8[1];
            r[3][0] = g0[2]; r[3][1] = g8[2]; r[3][2] = g0[3]; r[3][3] = g8[3];
        } else {
            // words: x = row g k0..15, y = row g+8 k0..15
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                r[s][0] = dequant_t2_pair<kBF16>(w.x, 2 * s);
                r[s][1] = dequant_t2_pair<kBF16>(w.y, 2 * s);
                r[s][2] = dequant_t2_pair<kBF16>(w.x, 2 * s + 1);
                r[s][3] = dequant_t2_pair<kBF16>(w.y, 2 * s + 1);
            }
        }
    }
};

template <typename ST>
__device__ __forceinline__ float lds_scale(const uint8_t* sp) {
    return to_f32(*reinterpret_cast<const ST*>(sp));
}

}  // namespace frag
}  // namespace hq
