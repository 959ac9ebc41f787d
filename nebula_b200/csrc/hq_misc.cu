// hq_misc.cu -- the plain fp32 GEMM behind the engine shim's forward_reference.
//
// Same arithmetic as kernel_reference_gemm (hydrogen/src/model/marlin_gemm.cu:52-70):
// one output per thread, sum = fma(X[m][k], W[k][n], sum) for k ascending, so
// the result is bit-identical; tiles of X and W go through shared memory.
#include "hq_internal.h"

namespace hq {

namespace {

constexpr int kT = 32;

__global__ void f32_gemm_kernel(const float* __restrict__ X, const float* __restrict__ W, float* __restrict__ Y,
                                int M, int K, int N) {
    __shared__ float xs[kT][kT + 1];
    __shared__ float ws[kT][kT + 1];
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int n = blockIdx.x * kT + tx;
    const int m0 = blockIdx.y * kT;
    float acc[kT / 8];
#pragma unroll
    for (int i = 0; i < kT / 8; ++i) acc[i] = 0.f;
    for (int k0 = 0; k0 < K; k0 += kT) {
        for (int r = ty; r < kT; r += 8) {
            const int m = m0 + r, k = k0 + tx;
            xs[r][tx] = (m < M && k < K) ? X[(size_t)m * K + k] : 0.f;
            const int kk = k0 + r;
            ws[r][tx] = (kk < K && n < N) ? W[(size_t)kk * N + n] : 0.f;
        }
        __syncthreads();
        const int kmax = K - k0 < kT ? K - k0 : kT;
        for (int kk = 0; kk < kmax; ++kk) {
            const float w = ws[kk][tx];
#pragma unroll
            for (int i = 0; i < kT / 8; ++i) acc[i] = __fmaf_rn(xs[ty + 8 * i][kk], w, acc[i]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < kT / 8; ++i) {
        const int m = m0 + ty + 8 * i;
        if (m < M && n < N) Y[(size_t)m * N + n] = acc[i];
    }
}

// The un-optimised comparator behind MarlinGemmEngine::forward_baseline_int4.
// The reference defines that entry point as a scalar-load kernel on the linear
// layout, the yardstick its Marlin path is measured against
// (marlin_gemm.cu:72-117).  Here: one thread per output column, one 32-bit
// word of codes per load straight from global memory, w = u * s + b rounded
// after the product and after the sum as the reference's host dequant computes
// it (:506; (u - 8) * s without biases), fp32 FMA in k order, up to eight
// token rows per pass over K and as many passes as M needs.  The result is
// therefore bit-identical to kernel_reference_gemm (:52-70) applied to the
// dequantised weights.
__global__ void baseline_linear_u4_kernel(const float* __restrict__ X, const uint32_t* __restrict__ W,
                                          const float* __restrict__ S, const float* __restrict__ B,
                                          float* __restrict__ Y, int M, int K, int N, int group) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    for (int m0 = 0; m0 < M; m0 += 8) {
        const int rows = M - m0 < 8 ? M - m0 : 8;
        float acc[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r] = 0.f;
        for (int kw = 0; kw < K / 8; ++kw) {
            const uint32_t word = W[(size_t)kw * N + n];
            const size_t gi = (size_t)(kw * 8 / group) * N + n;
            const float s = S[gi];
            const float b = B ? B[gi] : 0.f;
            for (int i = 0; i < 8; ++i) {
                const uint32_t u = (word >> (4 * i)) & 0xFu;
                const float w = B ? __fadd_rn(__fmul_rn((float)u, s), b) : __fmul_rn((float)((int)u - 8), s);
                const float* x = X + (size_t)m0 * K + (size_t)kw * 8 + i;
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < rows) acc[r] = __fmaf_rn(x[(size_t)r * K], w, acc[r]);
            }
        }
        for (int r = 0; r < rows; ++r) Y[(size_t)(m0 + r) * N + n] = acc[r];
    }
}

}  // namespace

cudaError_t launch_baseline_u4(const float* X, const uint32_t* W, const float* S, const float* B, float* Y, int M,
                               int K, int N, int group, cudaStream_t s) {
    if (M < 1 || K < 8 || N < 1 || group < 8 || K % group || group % 8) return cudaErrorInvalidValue;
    baseline_linear_u4_kernel<<<(N + 127) / 128, 128, 0, s>>>(X, W, S, B, Y, M, K, N, group);
    return cudaGetLastError();
}

cudaError_t launch_f32_gemm(const float* X, const float* W, float* Y, int M, int K, int N, cudaStream_t s) {
    dim3 block(kT, 8);
    dim3 grid((N + kT - 1) / kT, (M + kT - 1) / kT);
    f32_gemm_kernel<<<grid, block, 0, s>>>(X, W, Y, M, K, N);
    return cudaGetLastError();
}

}  // namespace hq
