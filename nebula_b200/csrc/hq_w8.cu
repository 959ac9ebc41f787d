// hq_w8.cu -- the reference engine's third precision, the W8A8 path
// (MarlinGemmEngine::forward_cutlass_int8 -> kernel_cutlass_int8_gemm,
// marlin_gemm.cu:327-377, 603-617):
//   q8(x)   = (int8) trunc(clamp(x * 127, -128, 127))      (per element, :351-354)
//   Y[m][n] = scale[n] * sum over the K/4 whole quads of k of
//             dp4a(q8(X[m][4q..4q+3]), W[4q..4q+3][n]) / 127
// W is int8 [K][N] (k-major rows), scale fp32 [N], X and Y fp32 row-major.
//
// The reference keeps one fp32 running sum per (m, n) and rounds after every
// quad.  Here the dot products are summed exactly in int32 (|sum| <= K * 128^2
// < 2^31 for K < 2^17) and rounded once, so k can be split across CTAs.  One
// launch, w8_gemm_kernel: a thread-block cluster of up to 8 CTAs per column
// tile of 128, CTA r taking quad range r.  Each CTA quantizes its X quads into
// shared memory; each warp takes every 8th quad of the range, each lane 4
// columns (one 32-bit load per row, a 4x4 byte transpose by byte permutes, one
// dp4a per column and row of X); the 8 warps' int32 partials are summed in
// shared memory.  After a cluster barrier CTA r sums 1/cs of the tile over the
// cluster's CTAs through distributed shared memory (exact integers, so the
// order does not matter), applies (1/127) * scale and stores Y: no memset, no
// atomics, no second kernel.
#include "hq.h"
#include "hq_common.cuh"
#include "hq_internal.h"

namespace hq {

namespace {

constexpr int kW8Threads = 256;
constexpr int kW8Warps = kW8Threads / 32;
constexpr int kW8Cols = 128;      // columns per CTA: 32 lanes x 4
constexpr int kW8MaxM = 8;        // rows of X per launch
constexpr int kW8MaxQuads = 2048; // quads per CTA (shared-memory X quads: kW8MaxM x 8 KB)
constexpr int kW8MaxSplits = 8;   // CTAs per cluster (portable size)

// q8 of four consecutive activations, packed as int8 lanes (marlin_gemm.cu:351-360).
__device__ __forceinline__ uint32_t q8_quad(const float* x) {
    uint32_t r = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float v = fminf(fmaxf(x[i] * 127.0f, -128.0f), 127.0f);
        r |= ((uint32_t)(int)v & 0xFFu) << (8 * i);  // float -> int truncates toward zero, as static_cast does
    }
    return r;
}

__global__ void __launch_bounds__(kW8Threads) w8_gemm_kernel(const float* __restrict__ X,
                                                             const int8_t* __restrict__ W,
                                                             const float* __restrict__ scales,
                                                             float* __restrict__ Y, int M, int K, int N,
                                                             int quads_per_cta) {
    extern __shared__ uint32_t xq[];  // [M][quads_per_cta]
    __shared__ int red[kW8Warps][kW8MaxM][kW8Cols];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quads = K / 4;
    const int q0 = blockIdx.y * quads_per_cta;
    const int nq = min(quads_per_cta, quads - q0);
    for (int i = threadIdx.x; i < M * nq; i += kW8Threads) {
        const int m = i / nq, q = i % nq;
        xq[m * quads_per_cta + q] = q8_quad(X + (size_t)m * K + 4 * (q0 + q));
    }
    __syncthreads();

    const int c0 = blockIdx.x * kW8Cols + 4 * lane;  // this lane's 4 columns (N % 4 == 0)
    int acc[kW8MaxM][4];
#pragma unroll
    for (int m = 0; m < kW8MaxM; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0;
    if (c0 < N) {
        const uint32_t* Wc = reinterpret_cast<const uint32_t*>(W + c0);
        const size_t row_words = (size_t)N / 4;
#pragma unroll 2
        for (int q = warp; q < nq; q += kW8Warps) {
            const size_t k = 4 * (size_t)(q0 + q);
            const uint32_t r0 = __ldg(Wc + (k + 0) * row_words), r1 = __ldg(Wc + (k + 1) * row_words);
            const uint32_t r2 = __ldg(Wc + (k + 2) * row_words), r3 = __ldg(Wc + (k + 3) * row_words);
            // column c's quad = byte c of r0..r3
            const uint32_t t0 = __byte_perm(r0, r1, 0x5140), t1 = __byte_perm(r0, r1, 0x7362);
            const uint32_t t2 = __byte_perm(r2, r3, 0x5140), t3 = __byte_perm(r2, r3, 0x7362);
            const uint32_t col[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632),
                                     __byte_perm(t1, t3, 0x5410), __byte_perm(t1, t3, 0x7632)};
#pragma unroll
            for (int m = 0; m < kW8MaxM; ++m) {
                if (m < M) {
                    const int xm = (int)xq[m * quads_per_cta + q];
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[m][c] = __dp4a(xm, (int)col[c], acc[m][c]);
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kW8MaxM; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[warp][m][4 * lane + c] = acc[m][c];
    __syncthreads();
    // this CTA's partial tile into red[0] (each element read and written by one thread)
    for (int i = threadIdx.x; i < M * kW8Cols; i += kW8Threads) {
        const int m = i / kW8Cols, cc = i % kW8Cols;
        int s = 0;
#pragma unroll
        for (int w = 0; w < kW8Warps; ++w) s += red[w][m][cc];
        red[0][m][cc] = s;
    }
    const int cs = (int)gridDim.y;  // the cluster spans the k splits of this column tile
    const int rank = (int)blockIdx.y;
    cluster_sync();
    const int total = M * kW8Cols, share = (total + cs - 1) / cs;
    for (int i = rank * share + threadIdx.x; i < min(total, (rank + 1) * share); i += kW8Threads) {
        const int m = i / kW8Cols, cc = i % kW8Cols;
        const int col = blockIdx.x * kW8Cols + cc;
        const uint32_t a = smem_u32(&red[0][m][cc]);
        int s = 0;
        for (int r = 0; r < cs; ++r) {
            int v;
            asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(mapa_shared(a, (uint32_t)r)) : "memory");
            s += v;
        }
        if (col < N) Y[(size_t)m * N + col] = ((float)s * (1.0f / 127.0f)) * scales[col];
    }
    cluster_sync();  // every CTA's shared memory stays alive until the remote reads are done
}

}  // namespace

cudaError_t launch_w8_gemm(const float* X, const int8_t* W, const float* scales, float* Y, int M, int K, int N,
                           cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int quads = K / 4;
    const int col_tiles = (N + kW8Cols - 1) / kW8Cols;
    const int sms = device_info(dev).sm_count;
    // k splits per column tile: about two CTAs per SM in all, at least 64 quads each,
    // at most kW8MaxSplits (one cluster), each within the shared-memory X stage
    int splits = quads > 0 ? (2 * sms + col_tiles - 1) / col_tiles : 1;
    splits = max(1, min(splits, min(kW8MaxSplits, max(1, quads / 64))));
    splits = max(splits, (quads + kW8MaxQuads - 1) / kW8MaxQuads);
    const int qpc = quads > 0 ? (quads + splits - 1) / splits : 1;
    splits = quads > 0 ? (quads + qpc - 1) / qpc : 1;
    if (splits > kW8MaxSplits) return cudaErrorInvalidValue;  // K > 4 * kW8MaxQuads * kW8MaxSplits
    const size_t smem = (size_t)kW8MaxM * qpc * sizeof(uint32_t);
    e = ensure_smem_attr(reinterpret_cast<const void*>(w8_gemm_kernel), dev, (int)smem);
    if (e != cudaSuccess) return e;
    for (int m0 = 0; m0 < M; m0 += kW8MaxM) {
        const int mm = min(kW8MaxM, M - m0);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)col_tiles, (unsigned)splits);
        cfg.blockDim = dim3(kW8Threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = (unsigned)splits;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, w8_gemm_kernel, X + (size_t)m0 * K, W, scales, Y + (size_t)m0 * N, mm, K, N,
                               qpc);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace hq
