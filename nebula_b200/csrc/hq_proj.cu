// hq_proj.cu -- the output projection GEMV and the embedding row lookup over
// the GGML tensor types of the reference's forward pass (gguf_parser.hpp:33-64):
// F32, BF16, Q8_0 (here) and TQ1_0 (hq_tq1.cu).
//
// * proj_dense_kernel<F32 | BF16>: drop-in for the F32 / BF16 branches of
//   kernel_output_projection (forward_baseline.cu:193-204).  HBM-bound stream:
//   x staged once per CTA in shared memory, each warp takes 4 rows at a time and
//   its lanes read 16-byte chunks of all 4 (two chunks per row in flight), so
//   one shared-memory read of x serves 4 rows.  fp32 FMA per lane, warp sum.
// * proj_q8_0_kernel: the Q8_0 branch (:205-217).  Q8_0 blocks are 34 bytes
//   (fp16 d + 32 int8): each warp copies 32 block pairs (2176 contiguous,
//   16-byte aligned bytes) of 2 rows into its two-stage shared-memory buffer
//   with 16-byte cp.async, one step ahead; then each lane takes one pair
//   (68 bytes, 17 words: a word stride of 17 is bank-conflict free).  x is
//   held as four int8 pieces of a 28-bit fixed-point copy (scale 2^(e-27),
//   e = exponent of max|x|), so a block's sum over q * x is four exact integer
//   dot products, 4 lanes per dp4a, with no int8 -> float conversion; the
//   block's d scales the combined value.  An x holding NaN/Inf takes the
//   reference's float loop.
// * proj_generic_kernel: any other shape or alignment; one warp per row with
//   the reference's lane-strided loop.
// * embedding_kernel: kernel_embedding_lookup (forward_baseline.cu:55-109),
//   one thread per element.
#include "hq.h"
#include "hq_common.cuh"
#include "hq_internal.h"

namespace hq {

namespace {

constexpr int kProjThreads = 256;
constexpr int kProjWarps = kProjThreads / 32;
constexpr int kDenseRows = 4;  // rows per warp, dense kernels
constexpr int kQ8Rows = 2;     // rows per warp, Q8_0 kernel

enum ProjKind { kF32 = 0, kBF16 = 1 };

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Stage x (n floats) into shared memory; x 16-byte aligned takes 16-byte loads.
// swizzle: chunk c (4 floats) of 64-float group p goes to chunk p*16 + ((c%16) ^ (p%16)).
template <bool kSwizzle>
__device__ __forceinline__ void stage_x(const float* __restrict__ x, float4* xs4, int n) {
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int c = threadIdx.x; c < n / 4; c += blockDim.x) {
            const int dst = kSwizzle ? (c & ~15) | ((c & 15) ^ ((c >> 4) & 15)) : c;
            xs4[dst] = __ldg(x4 + c);
        }
    } else {
        float* xs = reinterpret_cast<float*>(xs4);
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const int c = i >> 2;
            const int dst = kSwizzle ? (c & ~15) | ((c & 15) ^ ((c >> 4) & 15)) : c;
            xs[dst * 4 + (i & 3)] = __ldg(x + i);
        }
    }
}

template <int kKind>
__global__ void __launch_bounds__(kProjThreads) proj_dense_kernel(const float* __restrict__ x,
                                                                  const uint8_t* __restrict__ w,
                                                                  float* __restrict__ out, int K, int N) {
    extern __shared__ float4 xs4[];
    stage_x<false>(x, xs4, K);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)K * (kKind == kF32 ? 4 : 2);
    const int nc = kKind == kF32 ? K / 4 : K / 8;  // 16-byte chunks per row
    for (int r0 = (blockIdx.x * kProjWarps + warp) * kDenseRows; r0 < N; r0 += gridDim.x * kProjWarps * kDenseRows) {
        const uint4* p[kDenseRows];
#pragma unroll
        for (int i = 0; i < kDenseRows; ++i)
            p[i] = reinterpret_cast<const uint4*>(w + (size_t)min(r0 + i, N - 1) * row_bytes);
        float acc[kDenseRows];
#pragma unroll
        for (int i = 0; i < kDenseRows; ++i) acc[i] = 0.f;
#pragma unroll 2
        for (int c = lane; c < nc; c += 32) {
            uint4 v[kDenseRows];
#pragma unroll
            for (int i = 0; i < kDenseRows; ++i) v[i] = __ldg(p[i] + c);
            if (kKind == kF32) {
                const float4 xv = xs4[c];
#pragma unroll
                for (int i = 0; i < kDenseRows; ++i) {
                    acc[i] = fmaf(__uint_as_float(v[i].x), xv.x, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].y), xv.y, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].z), xv.z, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].w), xv.w, acc[i]);
                }
            } else {  // bf16: the value's bits are the high half of an fp32 (forward_baseline.cu:200-202)
                const float4 xa = xs4[2 * c], xb = xs4[2 * c + 1];
#pragma unroll
                for (int i = 0; i < kDenseRows; ++i) {
                    acc[i] = fmaf(__uint_as_float(v[i].x << 16), xa.x, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].x & 0xFFFF0000u), xa.y, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].y << 16), xa.z, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].y & 0xFFFF0000u), xa.w, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].z << 16), xb.x, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].z & 0xFFFF0000u), xb.y, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].w << 16), xb.z, acc[i]);
                    acc[i] = fmaf(__uint_as_float(v[i].w & 0xFFFF0000u), xb.w, acc[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kDenseRows; ++i) acc[i] = warp_sum(acc[i]);
        if (lane == 0) {
#pragma unroll
            for (int i = 0; i < kDenseRows; ++i)
                if (r0 + i < N) out[r0 + i] = acc[i];
        }
    }
}

// int8 byte `byte` of w (stored as q ^ 0x80 = q + 128) -> exact fp32 q.
__device__ __forceinline__ float s8x_to_f32(uint32_t wx, uint32_t byte) {
    return __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u | byte)) - 8388736.0f;  // 2^23 + 128
}

__device__ __forceinline__ void cp_async16(uint32_t smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_dst), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

constexpr int kQ8PairsPerStep = 32;                 // one block pair per lane
constexpr int kQ8StepBytes = kQ8PairsPerStep * 68;  // 2176 B of one row
constexpr int kQ8StageBytes = kQ8Rows * kQ8StepBytes;

// x as four int8 pieces (K bytes each, piece-major), then per warp two stages of kQ8Rows x 2176 bytes.
__host__ __device__ inline size_t q8_smem_bytes(int K) {
    return (size_t)K * 4 + (size_t)kProjWarps * 2 * kQ8StageBytes;
}

// 16-byte chunk c of a piece array lives at chunk (c & ~7) | ((c & 7) ^ ((c >> 3) & 7)): the lanes of a
// warp read chunk 4 pr + r of their pairs pr, and the swizzle spreads those over all eight 16-byte bank groups.
__device__ __forceinline__ int q8_chunk_pos(int c) { return (c & ~7) | ((c & 7) ^ ((c >> 3) & 7)); }

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    return __dp4a((int)a, (int)b, c);  // signed x signed 8-bit lanes, 32-bit accumulate
}

// The reference's float loop for one row (forward_baseline.cu:205-217): the path for an x holding NaN/Inf.
__device__ float q8_row_float(const float* __restrict__ x, const uint8_t* __restrict__ row, int nb, int lane) {
    float acc = 0.f;
    for (int b = lane; b < nb; b += 32) {
        const uint8_t* blk = row + (size_t)b * 34;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        for (int j = 0; j < 32; ++j) acc = fmaf(d * (float)(int8_t)blk[2 + j], x[b * 32 + j], acc);
    }
    return warp_sum(acc);
}

__global__ void __launch_bounds__(kProjThreads) proj_q8_0_kernel(const float* __restrict__ x,
                                                                 const uint8_t* __restrict__ w,
                                                                 float* __restrict__ out, int K, int N) {
    extern __shared__ __align__(16) uint8_t q8_smem[];
    __shared__ uint32_t s_max[kProjWarps];
    __shared__ int s_bad[kProjWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)(K / 32) * 34;  // a multiple of 16 (K % 256 == 0)
    const int np = K / 64;                            // block pairs per row
    const int nj = (np + kQ8PairsPerStep - 1) / kQ8PairsPerStep;
    const int first = blockIdx.x * kProjWarps + warp, stride = gridDim.x * kProjWarps;  // row pairs
    const int n_rp = (N + kQ8Rows - 1) / kQ8Rows;
    const int my_rp = first < n_rp ? (n_rp - first + stride - 1) / stride : 0;
    const int n_steps = my_rp * nj;
    const uint32_t xq_s = smem_u32(q8_smem);  // piece p of x at xq_s + p * K
    const uint32_t stage0 = xq_s + (uint32_t)K * 4u + (uint32_t)(warp * 2 * kQ8StageBytes);

    // step s: row pair first + (s / nj) * stride, pairs [32 (s % nj), +32) of both rows, into stage s & 1
    auto issue = [&](int st) {
        if (st < n_steps) {
            const int rp = first + (st / nj) * stride, j = st % nj;
            const int pairs = min(kQ8PairsPerStep, np - j * kQ8PairsPerStep);
            const int chunks = pairs * 68 / 16;  // pairs % 4 == 0
#pragma unroll
            for (int i = 0; i < kQ8Rows; ++i) {
                const uint8_t* src = w + (size_t)min(rp * kQ8Rows + i, N - 1) * row_bytes + (size_t)j * kQ8StepBytes;
                const uint32_t dst = stage0 + (st & 1) * kQ8StageBytes + i * kQ8StepBytes;
                for (int c = lane; c < chunks; c += 32) cp_async16(dst + 16 * c, src + 16 * c);
            }
        }
        cp_async_commit();  // one group per step, empty past the end
    };

    // 1. max|x| and finiteness; NaN/Inf in x -> the reference's float loop, row by row
    uint32_t m = 0;
    int bad = 0;
    for (int i = threadIdx.x; i < K; i += kProjThreads) {
        const float v = __ldg(x + i);
        bad |= !isfinite(v);
        m = max(m, __float_as_uint(fabsf(v)));
    }
    m = __reduce_max_sync(0xffffffffu, m);
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) s_max[warp] = m, s_bad[warp] = bad;
    __syncthreads();
    m = 0;
    bad = 0;
#pragma unroll
    for (int i = 0; i < kProjWarps; ++i) m = max(m, s_max[i]), bad |= s_bad[i];
    if (bad) {
        for (int rp = first; rp < n_rp; rp += stride)
            for (int i = 0; i < kQ8Rows; ++i) {
                const int row = rp * kQ8Rows + i;
                if (row >= N) break;
                const float v = q8_row_float(x, w + (size_t)row * row_bytes, K / 32, lane);
                if (lane == 0) out[row] = v;
            }
        return;
    }
    issue(0);
    issue(1);
    int e = 0;
    frexpf(__uint_as_float(m), &e);  // max|x| < 2^e (e = 0 when x == 0)

    // 2. x -> X = rint(x * 2^(27-e)) (|X| <= 2^27) as balanced base-128 digits q0..q3, piece-major int8
    for (int i = threadIdx.x; i < K; i += kProjThreads) {
        const int X = __float2int_rn(ldexpf(__ldg(x + i), 27 - e));
        const int q3 = ((X + 64) & 127) - 64;
        const int X1 = (X - q3) >> 7;
        const int q2 = ((X1 + 64) & 127) - 64;
        const int X2 = (X1 - q2) >> 7;
        const int q1 = ((X2 + 64) & 127) - 64;
        const int q0 = (X2 - q1) >> 7;
        const int pos = q8_chunk_pos(i >> 4) * 16 + (i & 15);
        q8_smem[0 * K + pos] = (uint8_t)q0;
        q8_smem[1 * K + pos] = (uint8_t)q1;
        q8_smem[2 * K + pos] = (uint8_t)q2;
        q8_smem[3 * K + pos] = (uint8_t)q3;
    }
    __syncthreads();

    // 3. per block and row: S_p = sum q * x_p (exact, 4 lanes per dp4a), value = (S0*128+S1) * 2^14 +
    //    (S2*128+S3), times the block's d; the row total is scaled by 2^(e-27) at the end.
    float acc[kQ8Rows];
#pragma unroll
    for (int i = 0; i < kQ8Rows; ++i) acc[i] = 0.f;
    for (int st = 0; st < n_steps; ++st) {
        const int rp = first + (st / nj) * stride, j = st % nj;
        cp_async_wait_1();  // this lane's copies of step st are done
        __syncwarp();       // ... and every lane's
        const int pr = j * kQ8PairsPerStep + lane;
        if (pr < np) {
            const uint32_t sp = stage0 + (st & 1) * kQ8StageBytes + lane * 68;  // word stride 17: no bank conflicts
            uint32_t W[kQ8Rows][17];
#pragma unroll
            for (int i = 0; i < kQ8Rows; ++i)
#pragma unroll
                for (int k = 0; k < 17; ++k)
                    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(W[i][k]) : "r"(sp + i * kQ8StepBytes + 4 * k));
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                uint4 xp[4][2];  // pieces 0..3 of the block's 32 x values
#pragma unroll
                for (int p = 0; p < 4; ++p)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                                     : "=r"(xp[p][h].x), "=r"(xp[p][h].y), "=r"(xp[p][h].z), "=r"(xp[p][h].w)
                                     : "r"(xq_s + (uint32_t)(p * K + q8_chunk_pos(4 * pr + 2 * blk + h) * 16)));
#pragma unroll
                for (int i = 0; i < kQ8Rows; ++i) {
                    uint32_t q[8];  // the block's 32 int8 weights, 4 per word
#pragma unroll
                    for (int g = 0; g < 8; ++g)
                        q[g] = blk == 0 ? __funnelshift_r(W[i][g], W[i][g + 1], 16) : W[i][9 + g];
                    int S[4];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const uint32_t xw[8] = {xp[p][0].x, xp[p][0].y, xp[p][0].z, xp[p][0].w,
                                                xp[p][1].x, xp[p][1].y, xp[p][1].z, xp[p][1].w};
                        S[p] = 0;
#pragma unroll
                        for (int g = 0; g < 8; ++g) S[p] = dp4a(q[g], xw[g], S[p]);
                    }
                    // |S_p| <= 32 * 128 * 65: S0*128 + S1 and S2*128 + S3 fit in int32 (one fp32 rounding each)
                    const float v = fmaf((float)(S[0] * 128 + S[1]), 16384.f, (float)(S[2] * 128 + S[3]));
                    const uint32_t dbits = blk == 0 ? (W[i][0] & 0xFFFFu) : (W[i][8] >> 16);
                    acc[i] = fmaf(__half2float(__ushort_as_half((unsigned short)dbits)), v, acc[i]);
                }
            }
        }
        __syncwarp();  // every lane is done with stage st & 1
        issue(st + 2);
        if (j == nj - 1) {  // row pair done
#pragma unroll
            for (int i = 0; i < kQ8Rows; ++i) {
                const float v = ldexpf(warp_sum(acc[i]), e - 27);
                if (lane == 0 && rp * kQ8Rows + i < N) out[rp * kQ8Rows + i] = v;
                acc[i] = 0.f;
            }
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// The reference's loop (forward_baseline.cu:193-217) for shapes and alignments
// the stream kernels do not take; x read from global memory.
__global__ void __launch_bounds__(kProjThreads) proj_generic_kernel(const float* __restrict__ x,
                                                                    const uint8_t* __restrict__ w, int type,
                                                                    float* __restrict__ out, int K, int N) {
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * kProjWarps + (threadIdx.x >> 5); row < N; row += gridDim.x * kProjWarps) {
        float acc = 0.f;
        if (type == HQ_GGML_F32) {
            const float* r = reinterpret_cast<const float*>(w) + (size_t)row * K;
            for (int i = lane; i < K; i += 32) acc = fmaf(r[i], x[i], acc);
        } else if (type == HQ_GGML_BF16) {
            const uint16_t* r = reinterpret_cast<const uint16_t*>(w) + (size_t)row * K;
            for (int i = lane; i < K; i += 32) acc = fmaf(__uint_as_float((uint32_t)r[i] << 16), x[i], acc);
        } else {  // Q8_0
            const int nb = K / 32;
            const uint8_t* r = w + (size_t)row * nb * 34;
            for (int b = lane; b < nb; b += 32) {
                const uint8_t* blk = r + (size_t)b * 34;
                const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
                for (int j = 0; j < 32; ++j) acc = fmaf(d * (float)(int8_t)blk[2 + j], x[b * 32 + j], acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) out[row] = acc;
    }
}

__global__ void embedding_kernel(const uint8_t* __restrict__ table, int type, int token_id, float* __restrict__ out,
                                 int K) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= K) return;
    if (type == HQ_GGML_F32) {
        out[i] = reinterpret_cast<const float*>(table)[(size_t)token_id * K + i];
    } else if (type == HQ_GGML_BF16) {
        out[i] = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(table)[(size_t)token_id * K + i] << 16);
    } else if (type == HQ_GGML_Q8_0) {
        const uint8_t* blk = table + ((size_t)token_id * (K / 32) + i / 32) * 34;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        out[i] = d * (float)(int8_t)blk[2 + i % 32];
    } else {  // TQ1_0 (native_decoder.cu:63-103): NaN/Inf d -> 0
        const uint8_t* blk = table + ((size_t)token_id * (K / 256) + i / 256) * 56;
        float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        if (isnan(d) || isinf(d)) d = 0.f;
        const int e = i % 256;
        uint32_t v = e < 250 ? blk[2 + e / 5] : blk[52 + (e - 250) / 3];
        const int s = e < 250 ? e % 5 : (e - 250) % 3;
        for (int k = 0; k < s; ++k) v /= 3u;
        out[i] = d * (float)((int)(v % 3u) - 1);
    }
}

cudaError_t launch_stream_kernel(const void* fn, const float* x, const uint8_t* w, float* out, int K, int N,
                                 int rows_per_warp, size_t smem, cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(fn, dev, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kProjThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    const int want = (N + kProjWarps * rows_per_warp - 1) / (kProjWarps * rows_per_warp);
    const int cap = device_info(dev).sm_count * per_sm;
    const int grid = want < cap ? want : cap;
    void* args[] = {(void*)&x, (void*)&w, (void*)&out, (void*)&K, (void*)&N};
    return cudaLaunchKernel(fn, grid, kProjThreads, args, smem, s);
}

}  // namespace

cudaError_t launch_output_projection(const float* x, const uint8_t* w, int type, float* out, int K, int N,
                                     cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)K * sizeof(float);
    const bool x_fits = smem + 4096 <= device_info(dev).smem_optin;
    const uintptr_t wa = reinterpret_cast<uintptr_t>(w);
    if (type == HQ_GGML_F32 && x_fits && K % 4 == 0 && (wa & 15u) == 0)
        return launch_stream_kernel(reinterpret_cast<const void*>(proj_dense_kernel<kF32>), x, w, out, K, N,
                                    kDenseRows, smem, s);
    if (type == HQ_GGML_BF16 && x_fits && K % 8 == 0 && (wa & 15u) == 0)
        return launch_stream_kernel(reinterpret_cast<const void*>(proj_dense_kernel<kBF16>), x, w, out, K, N,
                                    kDenseRows, smem, s);
    if (type == HQ_GGML_Q8_0 && q8_smem_bytes(K) + 4096 <= device_info(dev).smem_optin && K % 256 == 0 &&
        (wa & 15u) == 0)
        return launch_stream_kernel(reinterpret_cast<const void*>(proj_q8_0_kernel), x, w, out, K, N, kQ8Rows,
                                    q8_smem_bytes(K), s);
    const int blocks = (N + kProjWarps - 1) / kProjWarps;
    const int grid = blocks < device_info(dev).sm_count * 16 ? blocks : device_info(dev).sm_count * 16;
    proj_generic_kernel<<<grid, kProjThreads, 0, s>>>(x, w, type, out, K, N);
    return cudaGetLastError();
}

cudaError_t launch_embedding_lookup(const uint8_t* table, int type, int token_id, float* out, int K, cudaStream_t s) {
    embedding_kernel<<<(K + 255) / 256, 256, 0, s>>>(table, type, token_id, out, K);
    return cudaGetLastError();
}

}  // namespace hq
