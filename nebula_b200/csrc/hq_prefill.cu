// hq_prefill.cu -- tensor-core (tcgen05 / TMEM) W4A16 / ternary GEMM for M > 16.
//
// The reference has no prefill GEMM (its decoder feeds the prompt one token at
// a time, hydrogen/src/model/native_decoder.cu:1297); this kernel is the
// B200 counterpart of the M >= 64 row of the quantized linear layer.
//
// One persistent CTA per SM walks output tiles of 128 tokens x 256 columns
// (m-fastest, so the CTAs in flight share each n-tile's weights through L2):
//   warp 4      producer: per 64-k block, a TMA box of the activations
//               (128 x 64, 128-byte swizzle), the packed weights of the tile's
//               two strip groups (1-D bulk copies of the tile order) and the
//               group-scale row of the 256 columns, into a 4-stage ring;
//   warps 6-13  dequantisers: each lane expands its 16 packed bytes (exact
//               integer codes via the exponent-OR trick), multiplies by the
//               column's group scale (16-bit packed mul) and stores 8-k
//               vectors into the K-major 128B-swizzled B tile of a 3-stage
//               ring, then fences the async proxy;
//   warp 5      one thread issues tcgen05.mma (M=128, N=256, K=16, fp32
//               accumulate in TMEM) and commits completions to the barriers;
//               the warp also allocates / frees the 512 TMEM columns that hold
//               two accumulators, so the epilogue of one tile overlaps the
//               main loop of the next;
//   warps 0-3   epilogue: tcgen05.ld of their 32 TMEM lanes (token rows),
//               conversion and 64-byte row-segment stores of C.
// Every barrier wait is bounded (see hq_common.cuh); nothing is allocated.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"
#include "hq_tmap.h"

#include <algorithm>
#include <cstring>
#include <type_traits>

namespace hq {

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kEpiWarps = 4;  // warps 0..3 (TMEM lane quarters)
constexpr int kProdWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kDqWarp0 = 6;
constexpr int kDqWarps = 8;  // warps 6..13, two 16-column strips each
constexpr int kThreads = (kDqWarp0 + kDqWarps) * 32;
constexpr int kS1 = 4;  // activation + packed-weight + scale stages
constexpr int kS2 = 3;  // dequantized weight stages
constexpr uint32_t kTmemCols = 512;

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

template <int WBITS>
struct PLayout {
    static constexpr int kCB = WBITS == 4 ? 512 : 256;
    static constexpr int kA = BM * BK * 2;                     // activation tile
    static constexpr int kPacked = (BN / kStripCols) * kCB;    // 16 chunks
    static constexpr int kScale = BN * 2;                      // 16-bit scales
    static constexpr int kS1Bytes = align_up(kA + kPacked + kScale, 1024);
    static constexpr int kB = BN * BK * 2;                     // dequantized weight tile
    static constexpr int kOffB = kS1 * kS1Bytes;
    static constexpr int kOffBar = kOffB + kS2 * kB;
    static constexpr int kSmem = kOffBar + 256 + 1024;         // barriers + TMEM slot + alignment slack
};

struct alignas(64) PrefillParams {
    CUtensorMap a_map;  // [M][K] 16-bit: box 64 x 128, 128B swizzle, rows >= M read zero
    const uint8_t* W;
    const void* S;
    void* C;
    unsigned* err;
    int M, N, K, group;
    int m_tiles, n_tiles;
};

template <typename T>
__device__ __forceinline__ uint32_t scale_pair(const uint8_t* sp) {
    const uint32_t v = *reinterpret_cast<const uint16_t*>(sp);
    return v | (v << 16);
}

template <bool kBF16>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t s) {
    return kBF16 ? bf16x2_mul(a, s) : hmul2_bits(a, s);
}

template <typename OT>
__device__ __forceinline__ void store_row(OT* dst, const uint32_t (&v)[32], int ncols);

template <>
__device__ __forceinline__ void store_row<float>(float* dst, const uint32_t (&v)[32], int ncols) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (4 * i < ncols)
            *reinterpret_cast<uint4*>(dst + 4 * i) = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

template <typename T16>
__device__ __forceinline__ void store_row16(T16* dst, const uint32_t (&v)[32], int ncols) {
    uint32_t h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        if constexpr (std::is_same<T16, __half>::value) {
            __half2 x = __floats2half2_rn(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            h[i] = *reinterpret_cast<uint32_t*>(&x);
        } else {
            __nv_bfloat162 x = __floats2bfloat162_rn(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
            h[i] = *reinterpret_cast<uint32_t*>(&x);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
        if (8 * i < ncols)
            *reinterpret_cast<uint4*>(dst + 8 * i) = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
}
template <>
__device__ __forceinline__ void store_row<__half>(__half* dst, const uint32_t (&v)[32], int ncols) {
    store_row16(dst, v, ncols);
}
template <>
__device__ __forceinline__ void store_row<__nv_bfloat16>(__nv_bfloat16* dst, const uint32_t (&v)[32], int ncols) {
    store_row16(dst, v, ncols);
}

template <int WBITS, typename T, typename OT>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
    using L = PLayout<WBITS>;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr int kCB = L::kCB;
    constexpr uint32_t kIdesc = umma_idesc_f16(kBF16, BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* ld_full = reinterpret_cast<uint64_t*>(sm + L::kOffBar);
    uint64_t* ld_empty = ld_full + kS1;
    uint64_t* b_full = ld_empty + kS1;
    uint64_t* b_empty = b_full + kS2;
    uint64_t* acc_full = b_empty + kS2;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WBITS);
    const int KB = geo.KB;
    const int num_tiles = p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kS1; ++i) {
            mbar_init(&ld_full[i], 1);
            mbar_init(&ld_empty[i], 1 + kDqWarps);
        }
        for (int i = 0; i < kS2; ++i) {
            mbar_init(&b_full[i], kDqWarps);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        fence_mbarrier_init();
        fence_async_smem();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_last();  // an n-tile's weights are re-read by every m-tile
            const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
            int kbc = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
                const int m0 = mt * BM, n0 = nt * BN;
                const int sg0 = n0 / kGroupCols;
                const int w0 = geo.width(sg0);
                const int w1 = sg0 + 1 < geo.NSG ? geo.width(sg0 + 1) : 0;
                const int ncols = p.N - n0 < BN ? p.N - n0 : BN;
                for (int kb = 0; kb < KB; ++kb, ++kbc) {
                    const int s = kbc % kS1;
                    if (!mbar_wait(&ld_empty[s], ((uint32_t)(kbc / kS1) & 1u) ^ 1u, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm + s * L::kS1Bytes;
                    const uint32_t bytes = (uint32_t)(L::kA + (w0 + w1) * kCB + ncols * 2);
                    mbar_arrive_expect_tx(&ld_full[s], bytes);
                    tma_load_2d(st, &p.a_map, kb * BK, m0, &ld_full[s]);
                    bulk_g2s_evict_first(st + L::kA, p.W + geo.unit_offset((long long)sg0 * KB + kb), w0 * kCB,
                                         &ld_full[s], pol);
                    if (w1)
                        bulk_g2s_evict_first(st + L::kA + kGroupStrips * kCB,
                                             p.W + geo.unit_offset((long long)(sg0 + 1) * KB + kb), w1 * kCB,
                                             &ld_full[s], pol);
                    const int gi = kb * BK / p.group;
                    bulk_g2s(st + L::kA + L::kPacked, Sb + ((size_t)gi * p.N + n0) * 2, ncols * 2, &ld_full[s]);
                }
            }
            // Loads still in flight land before the CTA exits.
            for (int k = kbc - kS1 < 0 ? 0 : kbc - kS1; k < kbc; ++k)
                mbar_wait(&ld_full[k % kS1], (uint32_t)(k / kS1) & 1u, p.err);
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ----------------------------------------------------------- MMA issue
        if (lane == 0) {
            int kbc = 0, tc = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
                const int b = tc & 1;
                if (ok) ok = mbar_wait(&acc_empty[b], ((uint32_t)(tc >> 1) & 1u) ^ 1u, p.err);
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
                for (int kb = 0; kb < KB; ++kb, ++kbc) {
                    const int s1 = kbc % kS1, s2 = kbc % kS2;
                    if (ok) ok = mbar_wait(&ld_full[s1], (uint32_t)(kbc / kS1) & 1u, p.err);
                    if (ok) ok = mbar_wait(&b_full[s2], (uint32_t)(kbc / kS2) & 1u, p.err);
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sm + s1 * L::kS1Bytes);
                    const uint32_t b_addr = smem_u32(sm + L::kOffB + s2 * L::kB);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_f16(d_tmem, sw128_kmajor_desc(a_addr + 32 * k), sw128_kmajor_desc(b_addr + 32 * k),
                                 kIdesc, (kb | k) != 0);
                    umma_commit(&ld_empty[s1]);
                    umma_commit(&b_empty[s2]);
                }
                umma_commit(&acc_full[b]);
            }
        }
        __syncwarp();
    } else if (warp >= kDqWarp0) {
        // ------------------------------------------------------- dequantisers
        const int dw = warp - kDqWarp0;
        const int g = lane >> 2, t = lane & 3;
        int kbc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int nt = tile / p.m_tiles;
            const int n0 = nt * BN;
            const int sg0 = n0 / kGroupCols;
            const int w0 = geo.width(sg0);
            const int w1 = sg0 + 1 < geo.NSG ? geo.width(sg0 + 1) : 0;
            for (int kb = 0; kb < KB; ++kb, ++kbc) {
                const int s1 = kbc % kS1, s2 = kbc % kS2;
                if (ok) ok = mbar_wait(&ld_full[s1], (uint32_t)(kbc / kS1) & 1u, p.err);
                if (ok) ok = mbar_wait(&b_empty[s2], ((uint32_t)(kbc / kS2) & 1u) ^ 1u, p.err);
                const uint8_t* packed = sm + s1 * L::kS1Bytes + L::kA;
                const uint8_t* scales = packed + L::kPacked;
                uint8_t* bt = sm + L::kOffB + s2 * L::kB;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int c = 2 * dw + cc;  // strip within the tile, 0..15
                    const int gs = c / kGroupStrips, sl = c % kGroupStrips;
                    if (sl >= (gs ? w1 : w0)) continue;
                    const uint8_t* src = packed + (gs * kGroupStrips + sl) * kCB + lane * (kCB / 32);
                    const int r0 = c * kStripCols + g, r1 = r0 + 8;  // B-tile rows (output columns)
                    const uint32_t sp0 = scale_pair<T>(scales + r0 * 2);
                    const uint32_t sp1 = scale_pair<T>(scales + r1 * 2);
                    uint32_t v0[8], v1[8];  // rows r0 / r1: k = 16t .. 16t+15 as 8 packed pairs
                    if constexpr (WBITS == 4) {
                        const uint4 w = *reinterpret_cast<const uint4*>(src);
                        uint32_t o[4];
                        if constexpr (kBF16) dequant_u4_bf16(w.x, o); else dequant_u4_f16(w.x, o);
#pragma unroll
                        for (int i = 0; i < 4; ++i) v0[i] = mul2<kBF16>(o[i], sp0);
                        if constexpr (kBF16) dequant_u4_bf16(w.y, o); else dequant_u4_f16(w.y, o);
#pragma unroll
                        for (int i = 0; i < 4; ++i) v0[4 + i] = mul2<kBF16>(o[i], sp0);
                        if constexpr (kBF16) dequant_u4_bf16(w.z, o); else dequant_u4_f16(w.z, o);
#pragma unroll
                        for (int i = 0; i < 4; ++i) v1[i] = mul2<kBF16>(o[i], sp1);
                        if constexpr (kBF16) dequant_u4_bf16(w.w, o); else dequant_u4_f16(w.w, o);
#pragma unroll
                        for (int i = 0; i < 4; ++i) v1[4 + i] = mul2<kBF16>(o[i], sp1);
                    } else {
                        const uint2 w = *reinterpret_cast<const uint2*>(src);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            v0[i] = mul2<kBF16>(dequant_t2_pair<kBF16>(w.x, i), sp0);
                            v1[i] = mul2<kBF16>(dequant_t2_pair<kBF16>(w.y, i), sp1);
                        }
                    }
                    // 128B-swizzled K-major rows: 16-byte chunk q of row r at ((q ^ (r & 7)) << 4).
                    uint8_t* row0 = bt + r0 * 128;
                    uint8_t* row1 = bt + r1 * 128;
                    *reinterpret_cast<uint4*>(row0 + (((2 * t) ^ (r0 & 7)) << 4)) = make_uint4(v0[0], v0[1], v0[2], v0[3]);
                    *reinterpret_cast<uint4*>(row0 + (((2 * t + 1) ^ (r0 & 7)) << 4)) =
                        make_uint4(v0[4], v0[5], v0[6], v0[7]);
                    *reinterpret_cast<uint4*>(row1 + (((2 * t) ^ (r1 & 7)) << 4)) = make_uint4(v1[0], v1[1], v1[2], v1[3]);
                    *reinterpret_cast<uint4*>(row1 + (((2 * t + 1) ^ (r1 & 7)) << 4)) =
                        make_uint4(v1[4], v1[5], v1[6], v1[7]);
                }
                fence_async_smem();  // generic-proxy stores -> visible to the tensor core
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&b_full[s2]);
                    mbar_arrive(&ld_empty[s1]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        OT* C = reinterpret_cast<OT*>(p.C);
        int tc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int m0 = mt * BM, n0 = nt * BN;
            const int b = tc & 1;
            if (ok) ok = mbar_wait(&acc_full[b], (uint32_t)(tc >> 1) & 1u, p.err);
            tc_fence_after();
            const int row = m0 + 32 * warp + lane;
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * warp) << 16) + (uint32_t)(b * BN);
#pragma unroll 1
            for (int cb = 0; cb < BN / 32; ++cb) {
                uint32_t v[32];
                tmem_ld32(taddr + 32 * cb, v);
                tmem_ld_wait();
                const int col = n0 + 32 * cb;
                const int ncols = p.N - col < 32 ? p.N - col : 32;
                if (row < p.M && ncols > 0) store_row<OT>(C + (size_t)row * p.N + col, v, ncols);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }

    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

using PrefillFn = void (*)(PrefillParams);

template <int WBITS, typename T>
PrefillFn pick_out(DType c) {
    if (c == DType::F32) return prefill_kernel<WBITS, T, float>;
    if (std::is_same<T, __half>::value && c == DType::F16) return prefill_kernel<WBITS, T, __half>;
    if (std::is_same<T, __nv_bfloat16>::value && c == DType::BF16) return prefill_kernel<WBITS, T, __nv_bfloat16>;
    return nullptr;
}

PrefillFn select(const GemmArgs& a) {
    if (a.bias || a.s_dtype != a.a_dtype) return nullptr;
    if (a.a_dtype == DType::F16) return a.wbits == 4 ? pick_out<4, __half>(a.c_dtype) : pick_out<2, __half>(a.c_dtype);
    if (a.a_dtype == DType::BF16)
        return a.wbits == 4 ? pick_out<4, __nv_bfloat16>(a.c_dtype) : pick_out<2, __nv_bfloat16>(a.c_dtype);
    return nullptr;
}

}  // namespace

size_t prefill_workspace_bytes(int, int, int, int, int) { return 0; }

bool prefill_supported(const GemmArgs& a) { return select(a) != nullptr; }

cudaError_t launch_prefill(const GemmArgs& a) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    PrefillFn fn = select(a);
    if (!fn) return cudaErrorInvalidValue;
    const int smem = a.wbits == 4 ? PLayout<4>::kSmem : PLayout<2>::kSmem;
    e = ensure_smem_attr(reinterpret_cast<const void*>(fn), dev, smem);
    if (e != cudaSuccess) return e;
    PrefillParams p;
    memset(&p, 0, sizeof p);
    e = make_tmap_2d(&p.a_map, a.A, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2,
                     BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    p.W = a.W;
    p.S = a.S;
    p.C = a.C;
    p.err = device_error_word(dev);
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.group = a.group;
    p.m_tiles = (a.M + BM - 1) / BM;
    p.n_tiles = (a.N + BN - 1) / BN;
    const int tiles = p.m_tiles * p.n_tiles;
    const int grid = std::min(tiles, device_info(dev).sm_count);
    fn<<<grid, kThreads, smem, a.stream>>>(p);
    return cudaGetLastError();
}

}  // namespace hq
