// hq_tq1.cu -- TQ1_0 (the reference's base-3 ternary block) kernels.
//
// TQ1_0 block (hydrogen/src/model/native_decoder.cu:32-36): fp16 d, packed[52]
// (bytes 0..49 hold 5 trits, bytes 50..51 hold 3, least significant first,
// trit = digit - 1), 2 pad bytes = 56 bytes per 256 weights; rows of
// in_dim/256 blocks.
//
// * tq1_0_gemv: drop-in for kernel_gemv_tq1_0 (:155-206) at M = 1 with fp32 x.
//   One warp per output row (all rows computed, unlike the reference launch
//   at :1090-1091), each lane loads 8 contiguous bytes of the row (4 blocks per
//   warp pass), x staged once per CTA in shared memory, byte -> digits through
//   a shared 256-entry table.
// * tq1_0_to_tile_t2: offline conversion into this library's 2-bit tile order
//   so that the fast decode / tensor-core kernels run ternary weights.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"

namespace hq {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvRowsPerCta = kGemvThreads / 32;

// Digits 0..4 of byte v in base 3, 2 bits each (the same digit arithmetic as
// native_decoder.cu:183-186 for every byte value, including v >= 243).
__device__ __forceinline__ uint32_t base3_digits(uint32_t v) {
    uint32_t d = 0;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        d |= (v % 3u) << (2 * s);
        v /= 3u;
    }
    return d;
}

__device__ __forceinline__ float trit_times(uint32_t code, float x) {
    // code 0 -> -x, 1 -> 0, 2 -> +x
    return code == 2u ? x : (code == 0u ? -x : 0.0f);
}

__global__ void __launch_bounds__(kGemvThreads) tq1_0_gemv_kernel(const float* __restrict__ x,
                                                                  const uint8_t* __restrict__ w,
                                                                  float* __restrict__ out, int in_dim,
                                                                  int out_dim) {
    extern __shared__ float sx[];
    __shared__ uint16_t lut[256];
    for (int i = threadIdx.x; i < in_dim; i += blockDim.x) sx[i] = x[i];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = (uint16_t)base3_digits((uint32_t)i);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = in_dim / 256;
    const int blk_in_pass = lane / 7, part = lane % 7;  // lanes 0..27 active
    for (int row = blockIdx.x * kGemvRowsPerCta + warp; row < out_dim; row += gridDim.x * kGemvRowsPerCta) {
        const uint8_t* rowp = w + (size_t)row * nb * 56;
        float sum = 0.f;
        for (int b0 = 0; b0 < nb; b0 += 4) {
            const int b = b0 + blk_in_pass;
            float part_sum = 0.f;
            float d = 0.f;
            bool active = lane < 28 && b < nb;
            uint2 v = make_uint2(0, 0);
            if (active) v = __ldg(reinterpret_cast<const uint2*>(rowp + (size_t)b * 56 + part * 8));
            // d lives in bytes 0-1 of the block = low half of lane part 0's first word
            const int src_lane = blk_in_pass * 7;
            const uint32_t dbits = __shfl_sync(0xffffffffu, v.x, src_lane < 32 ? src_lane : 0);
            if (active) {
                d = __half2float(__ushort_as_half((unsigned short)(dbits & 0xFFFFu)));
                const float* xp = sx + b * 256;
                uint8_t bytes[8];
                *reinterpret_cast<uint2*>(bytes) = v;
                // block byte offset of bytes[0] is 8*part; packed index = offset - 2
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int pi = 8 * part + i - 2;  // packed index
                    if (pi < 0 || pi > 51) continue;
                    const uint32_t dig = lut[bytes[i]];
                    if (pi < 50) {
#pragma unroll
                        for (int s = 0; s < 5; ++s) part_sum += trit_times((dig >> (2 * s)) & 3u, xp[pi * 5 + s]);
                    } else {
#pragma unroll
                        for (int s = 0; s < 3; ++s)
                            part_sum += trit_times((dig >> (2 * s)) & 3u, xp[250 + (pi - 50) * 3 + s]);
                    }
                }
                if (isnan(d) || isinf(d)) part_sum = 0.f, d = 0.f;  // native_decoder.cu:174
            }
            sum = fmaf(d, part_sum, sum);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, off);
        if (lane == 0) out[row] = sum;
    }
}

// One thread per tile word (s, kb, lane, j) + the scale array.
__global__ void tq1_0_to_tile_t2_kernel(const uint8_t* __restrict__ w, uint32_t* __restrict__ tile,
                                        uint16_t* __restrict__ scales, int K, int N) {
    const TileGeom geo(K, N, 2);
    const int nb = K / 256;
    const size_t total = geo.bytes() / 4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += stride) {
        const size_t chunk = i / 64;
        const int within = (int)(i % 64);
        const int lane = within / 2, j = within % 2;
        const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
        const int sg = (int)(chunk / per_full_group);
        const size_t rem = chunk - (size_t)sg * per_full_group;
        const int wd = geo.width(sg);
        const int kb = (int)(rem / wd), sl = (int)(rem % wd);
        int col, kw;
        tile_word_source(2, sg * kGroupStrips + sl, kb, lane, j, &col, &kw);
        const int k0 = kw * 16;
        const uint8_t* blk = w + ((size_t)col * nb + k0 / 256) * 56;
        uint32_t lin = 0;
        for (int e = 0; e < 16; ++e) {
            const int el = (k0 % 256) + e;
            const int by = el < 250 ? el / 5 : 50 + (el - 250) / 3;
            const int dg = el < 250 ? el % 5 : (el - 250) % 3;
            uint32_t v = blk[2 + by];
            for (int s = 0; s < dg; ++s) v /= 3u;
            lin |= (v % 3u) << (2 * e);  // code = trit + 1
        }
        tile[i] = t2_linear_to_tile(lin);
    }
    const size_t ns = (size_t)(K / 128) * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ns; i += stride) {
        const int gi = (int)(i / N), n = (int)(i % N);
        const uint8_t* blk = w + ((size_t)n * nb + gi / 2) * 56;
        uint16_t d = (uint16_t)(blk[0] | (blk[1] << 8));
        if ((d & 0x7C00u) == 0x7C00u) d = 0;  // NaN/Inf block: contributes nothing
        scales[i] = d;
    }
}

}  // namespace

cudaError_t launch_tq1_0_gemv(const float* x, const uint8_t* w, float* out, int in_dim, int out_dim,
                              cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)in_dim * sizeof(float);
    e = ensure_smem_attr(reinterpret_cast<const void*>(tq1_0_gemv_kernel), dev, (int)smem);
    if (e != cudaSuccess) return e;
    const int blocks_needed = (out_dim + kGemvRowsPerCta - 1) / kGemvRowsPerCta;
    const int grid = blocks_needed < device_info(dev).sm_count * 8 ? blocks_needed : device_info(dev).sm_count * 8;
    tq1_0_gemv_kernel<<<grid, kGemvThreads, smem, s>>>(x, w, out, in_dim, out_dim);
    return cudaGetLastError();
}

cudaError_t launch_tq1_0_to_tile_t2(const uint8_t* w, uint8_t* tile, uint16_t* scales, int K, int N,
                                    cudaStream_t s) {
    const TileGeom geo(K, N, 2);
    size_t total = geo.bytes() / 4;
    int grid = (int)((total + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    tq1_0_to_tile_t2_kernel<<<grid, 256, 0, s>>>(w, reinterpret_cast<uint32_t*>(tile), scales, K, N);
    return cudaGetLastError();
}

}  // namespace hq
