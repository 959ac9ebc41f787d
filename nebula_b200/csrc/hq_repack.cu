// hq_repack.cu -- bit-exact weight repacks between the reference layouts and the
// tile order, on device (one thread per output word, coalesced writes) and on
// host threads.  The reference's own repack is host-only and single-threaded
// (hydrogen/src/model/marlin_gemm.cu:432-467; its OpenMP pragma is inert because
// hydrogen/CMakeLists.txt never enables OpenMP).
#include "hq_internal.h"
#include "hq_layout.h"

#include <algorithm>
#include <thread>
#include <vector>

namespace hq {

namespace {

// Linear word (kw, n) of the reference linear layout or of the Marlin quad layout.
__device__ __forceinline__ uint32_t load_linear_word(const uint32_t* src, bool quad, int kw, int n, int N) {
    if (!quad) return __ldg(src + (size_t)kw * N + n);
    // quad (kq, n) word j = linear word (4kq + j, n)   (marlin_gemm.cu:449-453)
    return __ldg(src + ((size_t)(kw >> 2) * N + n) * 4 + (kw & 3));
}

__global__ void linear_to_tile_kernel(const uint32_t* __restrict__ src, bool quad, int wbits,
                                      uint32_t* __restrict__ dst, int K, int N) {
    const TileGeom geo(K, N, wbits);
    const int words_per_lane = wbits == 4 ? 4 : 2;
    const size_t total = geo.bytes() / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        // Output word i -> (chunk, lane, j); chunks are walked in storage order.
        const size_t chunk = i / (size_t)(32 * words_per_lane);
        const int within = (int)(i % (size_t)(32 * words_per_lane));
        const int lane = within / words_per_lane, j = within % words_per_lane;
        // Storage order: sg-major, then kb, then strip-in-group.
        const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
        const int sg = (int)(chunk / per_full_group);
        const size_t rem = chunk - (size_t)sg * per_full_group;
        const int w = geo.width(sg);
        const int kb = (int)(rem / w), sl = (int)(rem % w);
        const int s = sg * kGroupStrips + sl;
        int col, kw;
        tile_word_source(wbits, s, kb, lane, j, &col, &kw);
        const uint32_t v = load_linear_word(src, quad, kw, col, N);
        dst[i] = wbits == 4 ? u4_linear_to_tile(v) : t2_linear_to_tile(v);
    }
}

__global__ void tile_to_linear_kernel(const uint32_t* __restrict__ src, int wbits, uint32_t* __restrict__ dst,
                                      int K, int N) {
    const TileGeom geo(K, N, wbits);
    const int words_per_lane = wbits == 4 ? 4 : 2;
    const size_t total = geo.bytes() / 4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t chunk = i / (size_t)(32 * words_per_lane);
        const int within = (int)(i % (size_t)(32 * words_per_lane));
        const int lane = within / words_per_lane, j = within % words_per_lane;
        const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
        const int sg = (int)(chunk / per_full_group);
        const size_t rem = chunk - (size_t)sg * per_full_group;
        const int w = geo.width(sg);
        const int kb = (int)(rem / w), sl = (int)(rem % w);
        const int s = sg * kGroupStrips + sl;
        int col, kw;
        tile_word_source(wbits, s, kb, lane, j, &col, &kw);
        const uint32_t v = __ldg(src + i);
        dst[(size_t)kw * N + col] = wbits == 4 ? u4_tile_to_linear(v) : t2_tile_to_linear(v);
    }
}

__global__ void linear_quad_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst, int K, int N,
                                   bool inverse) {
    const size_t total = (size_t)(K / 8) * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        // i indexes the quad layout: ((kq*N + n)*4 + j)  <->  linear (4kq + j, n)
        const int j = (int)(i & 3);
        const size_t qn = i >> 2;
        const int n = (int)(qn % N), kq = (int)(qn / N);
        const size_t li = (size_t)(4 * kq + j) * N + n;
        if (!inverse)
            dst[i] = __ldg(src + li);
        else
            dst[li] = __ldg(src + i);
    }
}

int grid_for(size_t total) {
    size_t b = (total + 255) / 256;
    return (int)std::min<size_t>(b, 148 * 16);
}

}  // namespace

cudaError_t launch_linear_to_tile(const void* src, bool src_is_quad, int wbits, uint8_t* dst, int K, int N,
                                  cudaStream_t s) {
    const TileGeom geo(K, N, wbits);
    linear_to_tile_kernel<<<grid_for(geo.bytes() / 4), 256, 0, s>>>(reinterpret_cast<const uint32_t*>(src),
                                                                    src_is_quad, wbits,
                                                                    reinterpret_cast<uint32_t*>(dst), K, N);
    return cudaGetLastError();
}

cudaError_t launch_tile_to_linear(const uint8_t* src, int wbits, uint32_t* dst, int K, int N, cudaStream_t s) {
    const TileGeom geo(K, N, wbits);
    tile_to_linear_kernel<<<grid_for(geo.bytes() / 4), 256, 0, s>>>(reinterpret_cast<const uint32_t*>(src), wbits,
                                                                    dst, K, N);
    return cudaGetLastError();
}

cudaError_t launch_linear_to_quad(const uint32_t* src, uint32_t* dst, int K, int N, bool inverse, cudaStream_t s) {
    linear_quad_kernel<<<grid_for((size_t)(K / 8) * N), 256, 0, s>>>(src, dst, K, N, inverse);
    return cudaGetLastError();
}

// ------------------------------------------------------------------- host

namespace host {

template <typename F>
void parallel_for(size_t n, int nthreads, F&& f) {
    if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
    nthreads = (int)std::min<size_t>((size_t)nthreads, std::max<size_t>(1, n / 4096));
    if (nthreads <= 1) {
        f((size_t)0, n);
        return;
    }
    std::vector<std::thread> th;
    th.reserve(nthreads);
    for (int t = 0; t < nthreads; ++t) {
        size_t a = n * t / nthreads, b = n * (t + 1) / nthreads;
        th.emplace_back([&f, a, b] { f(a, b); });
    }
    for (auto& x : th) x.join();
}

void linear_to_tile(const uint32_t* src, bool quad, int wbits, uint32_t* dst, int K, int N, int nthreads) {
    const TileGeom geo(K, N, wbits);
    const int wpl = wbits == 4 ? 4 : 2;
    const size_t total = geo.bytes() / 4;
    parallel_for(total, nthreads, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) {
            const size_t chunk = i / (size_t)(32 * wpl);
            const int within = (int)(i % (size_t)(32 * wpl));
            const int lane = within / wpl, j = within % wpl;
            const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
            const int sg = (int)(chunk / per_full_group);
            const size_t rem = chunk - (size_t)sg * per_full_group;
            const int w = geo.width(sg);
            const int kb = (int)(rem / w), sl = (int)(rem % w);
            int col, kw;
            tile_word_source(wbits, sg * kGroupStrips + sl, kb, lane, j, &col, &kw);
            const uint32_t v = quad ? src[((size_t)(kw >> 2) * N + col) * 4 + (kw & 3)] : src[(size_t)kw * N + col];
            dst[i] = wbits == 4 ? u4_linear_to_tile(v) : t2_linear_to_tile(v);
        }
    });
}

void tile_to_linear(const uint32_t* src, int wbits, uint32_t* dst, int K, int N, int nthreads) {
    const TileGeom geo(K, N, wbits);
    const int wpl = wbits == 4 ? 4 : 2;
    const size_t total = geo.bytes() / 4;
    parallel_for(total, nthreads, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) {
            const size_t chunk = i / (size_t)(32 * wpl);
            const int within = (int)(i % (size_t)(32 * wpl));
            const int lane = within / wpl, j = within % wpl;
            const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
            const int sg = (int)(chunk / per_full_group);
            const size_t rem = chunk - (size_t)sg * per_full_group;
            const int w = geo.width(sg);
            const int kb = (int)(rem / w), sl = (int)(rem % w);
            int col, kw;
            tile_word_source(wbits, sg * kGroupStrips + sl, kb, lane, j, &col, &kw);
            const uint32_t v = src[i];
            dst[(size_t)kw * N + col] = wbits == 4 ? u4_tile_to_linear(v) : t2_tile_to_linear(v);
        }
    });
}

// marlin_gemm.cu:446-455, parallel over kq (the reference's intended OpenMP split).
void linear_quad(const uint32_t* src, uint32_t* dst, int K, int N, bool inverse, int nthreads) {
    const size_t nkq = (size_t)K / 32;
    parallel_for(nkq * (size_t)N, nthreads, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) {
            const size_t kq = i / N, n = i % N;
            for (int j = 0; j < 4; ++j) {
                const size_t qi = (kq * N + n) * 4 + j, li = (kq * 4 + j) * N + n;
                if (!inverse)
                    dst[qi] = src[li];
                else
                    dst[li] = src[qi];
            }
        }
    });
}

}  // namespace host

}  // namespace hq
