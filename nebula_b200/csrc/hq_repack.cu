// hq_repack.cu -- bit-exact weight repacks between the reference layouts and the
// tile order, on device (one thread per output word, coalesced writes) and on
// host threads.  The reference's own repack is host-only and single-threaded
// (hydrogen/src/model/marlin_gemm.cu:432-467; its OpenMP pragma is inert because
// hydrogen/CMakeLists.txt never enables OpenMP).
#include "hq_internal.h"
#include "hq_layout.h"

#include <algorithm>
#include <cstring>
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
                                      uint32_t* __restrict__ dst, int K, int N, bool k32) {
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
        tile_word_source(wbits, s, kb, lane, j, &col, &kw, k32);
        const uint32_t v = load_linear_word(src, quad, kw, col, N);
        dst[i] = wbits == 4 ? u4_linear_to_tile(v) : t2_linear_to_tile(v);
    }
}

__global__ void tile_to_linear_kernel(const uint32_t* __restrict__ src, int wbits, uint32_t* __restrict__ dst,
                                      int K, int N, bool k32) {
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
        tile_word_source(wbits, s, kb, lane, j, &col, &kw, k32);
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

// ------------------------------------------------------------------ Q4_K
// GGUF Q4_K super-block: 256 weights of one row in 144 bytes (the block size
// hydrogen/include/gguf_parser.hpp:130 gives type 12; the field layout is
// llama.cpp's published block_q4_K, ggml/src/ggml-common.h):
//   bytes 0-1   fp16 d, bytes 2-3 fp16 dmin;
//   bytes 4-15  6-bit scale sc_i and min m_i of each 32-weight sub-block i;
//   bytes 16-143 codes: quarter j (64 weights) keeps k 64j + l in the low
//               nibble of byte 32j + l and k 64j + 32 + l in its high nibble.
// Weight = d * sc_i * u - dmin * m_i   (llama.cpp dequantize_row_q4_K), which
// is this library's biased form u * scale + bias with group 32, scale =
// d * sc_i and bias = -(dmin * m_i): both exact in fp32 (11 x 6 bits).
constexpr int kQ4KBlockBytes = 144;

// IEEE half bits -> float (normals, subnormals, Inf / NaN).
HQ_HD float half_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h >> 15) << 31;
    const int ex = (int)((h >> 10) & 31);
    uint32_t man = h & 0x3FFu, bits;
    if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (ex) {
        bits = sign | ((uint32_t)(ex + 112) << 23) | (man << 13);
    } else if (!man) {
        bits = sign;
    } else {  // subnormal: man * 2^-24, renormalised
        int e = 113;
        while (!(man & 0x400u)) {
            man <<= 1;
            --e;
        }
        bits = sign | ((uint32_t)e << 23) | ((man & 0x3FFu) << 13);
    }
#ifdef __CUDA_ARCH__
    return __uint_as_float(bits);
#else
    float f;
    memcpy(&f, &bits, 4);
    return f;
#endif
}

// Sub-block i (0..7) of the 12 packed bytes: i < 4 keeps sc / m in the low six
// bits of bytes i / i + 4; i >= 4 splits them over the low / high nibble of
// byte i + 4 and the top two bits of bytes i - 4 / i.
HQ_HD void q4k_scale_min(const uint8_t* p, int i, int* sc, int* m) {
    if (i < 4) {
        *sc = p[i] & 63;
        *m = p[i + 4] & 63;
    } else {
        *sc = (p[i + 4] & 0xF) | ((p[i - 4] >> 6) << 4);
        *m = (p[i + 4] >> 4) | ((p[i] >> 6) << 4);
    }
}

// The linear-order word (k0 + e at nibble e) of column `col`, k0 % 8 == 0: eight
// consecutive k sit in one half of one quarter, i.e. in 8 consecutive code bytes.
HQ_HD uint32_t q4k_linear_word(const uint8_t* w, int K, int col, int k0) {
    const uint8_t* blk = w + ((size_t)col * (size_t)(K / 256) + (size_t)(k0 / 256)) * kQ4KBlockBytes;
    const int within = k0 % 256, l = within % 64;
    const uint8_t* q = blk + 16 + 32 * (within / 64) + (l & 31);
    const int shift = l >= 32 ? 4 : 0;
    uint32_t lin = 0;
    for (int e = 0; e < 8; ++e) lin |= (uint32_t)((q[e] >> shift) & 0xF) << (4 * e);
    return lin;
}

// Scale and bias of (sub-block row g = k / 32, column n).
HQ_HD void q4k_scale_bias(const uint8_t* w, int K, int g, int n, float* scale, float* bias) {
    const uint8_t* blk = w + ((size_t)n * (size_t)(K / 256) + (size_t)(g / 8)) * kQ4KBlockBytes;
    int sc, m;
    q4k_scale_min(blk + 4, g % 8, &sc, &m);
    const float d = half_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    const float dmin = half_bits_to_f32((uint32_t)blk[2] | ((uint32_t)blk[3] << 8));
    *scale = d * (float)sc;
    *bias = -(dmin * (float)m);
}

// Tile word i (storage order, TILE_U4_K32) -> its column and first k.
HQ_HD void tile_word_coords(const TileGeom& geo, size_t i, int* col, int* k0) {
    const size_t chunk = i / 128;  // int4: 32 lanes x 4 words per chunk
    const int within = (int)(i % 128);
    const int lane = within / 4, j = within % 4;
    const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
    const int sg = (int)(chunk / per_full_group);
    const size_t rem = chunk - (size_t)sg * per_full_group;
    const int w = geo.width(sg);
    const int kb = (int)(rem / w), sl = (int)(rem % w);
    int kw;
    tile_word_source(4, sg * kGroupStrips + sl, kb, lane, j, col, &kw, true);
    *k0 = kw * 8;
}

__global__ void q4k_to_tile_kernel(const uint8_t* __restrict__ w, uint32_t* __restrict__ tile,
                                   float* __restrict__ scales, float* __restrict__ bias, int K, int N) {
    const TileGeom geo(K, N, 4);
    const size_t words = geo.bytes() / 4, rows = (size_t)(K / 32) * N;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words; i += stride) {
        int col, k0;
        tile_word_coords(geo, i, &col, &k0);
        tile[i] = u4_linear_to_tile(q4k_linear_word(w, K, col, k0));
    }
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < rows; i += stride) {
        const int n = (int)(i % N), g = (int)(i / N);  // n fastest: coalesced rows
        q4k_scale_bias(w, K, g, n, scales + i, bias + i);
    }
}

}  // namespace

cudaError_t launch_q4k_to_tile(const uint8_t* w, uint8_t* tile, float* scales, float* bias, int K, int N,
                               cudaStream_t s) {
    const TileGeom geo(K, N, 4);
    q4k_to_tile_kernel<<<grid_for(geo.bytes() / 4), 256, 0, s>>>(w, reinterpret_cast<uint32_t*>(tile), scales, bias,
                                                                 K, N);
    return cudaGetLastError();
}

cudaError_t launch_linear_to_tile(const void* src, bool src_is_quad, int wbits, uint8_t* dst, int K, int N,
                                  cudaStream_t s, bool k32) {
    const TileGeom geo(K, N, wbits);
    linear_to_tile_kernel<<<grid_for(geo.bytes() / 4), 256, 0, s>>>(reinterpret_cast<const uint32_t*>(src),
                                                                    src_is_quad, wbits,
                                                                    reinterpret_cast<uint32_t*>(dst), K, N, k32);
    return cudaGetLastError();
}

cudaError_t launch_tile_to_linear(const uint8_t* src, int wbits, uint32_t* dst, int K, int N, cudaStream_t s,
                                  bool k32) {
    const TileGeom geo(K, N, wbits);
    tile_to_linear_kernel<<<grid_for(geo.bytes() / 4), 256, 0, s>>>(reinterpret_cast<const uint32_t*>(src), wbits,
                                                                    dst, K, N, k32);
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

void linear_to_tile(const uint32_t* src, bool quad, int wbits, uint32_t* dst, int K, int N, int nthreads, bool k32) {
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
            tile_word_source(wbits, sg * kGroupStrips + sl, kb, lane, j, &col, &kw, k32);
            const uint32_t v = quad ? src[((size_t)(kw >> 2) * N + col) * 4 + (kw & 3)] : src[(size_t)kw * N + col];
            dst[i] = wbits == 4 ? u4_linear_to_tile(v) : t2_linear_to_tile(v);
        }
    });
}

void tile_to_linear(const uint32_t* src, int wbits, uint32_t* dst, int K, int N, int nthreads, bool k32) {
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
            tile_word_source(wbits, sg * kGroupStrips + sl, kb, lane, j, &col, &kw, k32);
            const uint32_t v = src[i];
            dst[(size_t)kw * N + col] = wbits == 4 ? u4_tile_to_linear(v) : t2_tile_to_linear(v);
        }
    });
}

void q4k_to_tile(const uint8_t* w, uint32_t* tile, float* scales, float* bias, int K, int N, int nthreads) {
    const TileGeom geo(K, N, 4);
    parallel_for(geo.bytes() / 4, nthreads, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) {
            int col, k0;
            tile_word_coords(geo, i, &col, &k0);
            tile[i] = u4_linear_to_tile(q4k_linear_word(w, K, col, k0));
        }
    });
    parallel_for((size_t)(K / 32) * N, nthreads, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) q4k_scale_bias(w, K, (int)(i / N), (int)(i % N), scales + i, bias + i);
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
