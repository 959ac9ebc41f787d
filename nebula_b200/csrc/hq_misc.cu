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

}  // namespace

cudaError_t launch_f32_gemm(const float* X, const float* W, float* Y, int M, int K, int N, cudaStream_t s) {
    dim3 block(kT, 8);
    dim3 grid((N + kT - 1) / kT, (M + kT - 1) / kT);
    f32_gemm_kernel<<<grid, block, 0, s>>>(X, W, Y, M, K, N);
    return cudaGetLastError();
}

}  // namespace hq
