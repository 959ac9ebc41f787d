// hq_decode_tc.cu -- decode GEMM (M <= 16) on the tcgen05 tensor cores.
//
// Replaces, for 16-bit activations and scales and scale groups that are
// multiples of 128, kernel_marlin_gemm_int4_templated / _dynamic and the
// memset + atomicAdd split-K of the reference
// (hydrogen/src/model/marlin_gemm.cu:130-322, :556-601).
//
// The weights are the M side of the MMA and live in tensor memory:
//   * Streaming as in the mma.sync decode kernel: a cluster of cs CTAs owns a
//     strip group (128 output columns); CTA r streams the group-aligned k range
//     [r G/cs, (r+1) G/cs) x group of it -- one contiguous byte span of the tile
//     order -- through a shared-memory ring: 1-D bulk copies for the codes, one
//     2-D TMA box (16 tokens x 64 k, 128B-swizzled, rows >= M zero) per k-block
//     for the activations, the group's scale row per stage.  A stage is two
//     k-blocks = 128 k inside one scale group.
//   * Eight dequant warps, two sets of four; set h expands k-block h of every
//     stage.  Warp q of a set owns TMEM lanes [32q, 32q+32) = output columns,
//     one column per thread: the thread gathers its column's 64 codes (four
//     8-byte loads from the lane fragments that hold them, start lane rotated
//     so a half-warp hits distinct banks), makes exact q
//     (exponent-OR plus one packed subtract per pair) and stores 32 packed
//     pairs to its set's A buffer with tcgen05.st.
//   * Two issuing threads (warps 9 and 10, one per set) issue, for their
//     k-block of each stage and each 16-k step, one M=128 x N=16 x K=16 MMA
//     (A from tensor memory, B = the activation tile's swizzled descriptor)
//     into the set's 16-column fp32 accumulator: four MMAs per 64 k each.
//     tcgen05.mma issue is the expensive step here (~100 cycles each
//     measured), hence exact q rather than a correction MMA, two issuers,
//     and one barrier wait per k-block on each.
//   * Each set drains its own accumulator one stage later (tcgen05.ld, times
//     the column's group scale in fp32, added in registers).  Because a warp
//     drains stage i-1 before it arrives for stage i+1, the arrival of a
//     set's four warps for a stage also proves that the A and D buffers it
//     reuses are free: the only waits are "stage landed" (dequant warps), "stage
//     expanded" (MMA thread), "stage accumulated" (drain) and "slot free"
//     (producer).
//   * Split-K partials (two sets x cs CTAs) are summed through distributed
//     shared memory in a fixed order; programmatic dependent launch with the
//     weights and scales requested before griddepcontrol.wait.
//   * At most two CTAs per SM (shared memory per CTA above a third of the
//     SM's), so the two 256-column tensor-memory allocations always fit and
//     tcgen05.alloc never waits on another CTA of the same launch.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"
#include "hq_tmap.h"

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

namespace hq {

namespace {

constexpr int kDqWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;  // issues set 0's MMAs and owns the TMEM allocation; warp 10 issues set 1's
constexpr int kThreads = 352;
constexpr int kStages = 6;  // shared-memory ring, two k-blocks per stage
constexpr int kTmemCols = 256;
// Tensor-memory map: A[set][buf] (32 columns each), D[set][buf] (16 columns each);
// two buffers of each suffice because a warp drains stage i-1 before it expands i+1.
constexpr uint32_t kColA = 0;
constexpr uint32_t kColD = 128;
constexpr int kMinSmem = 80 * 1024;  // > 1/3 of the SM's shared memory: at most two CTAs per SM
constexpr int kRows = 16;

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ constexpr uint32_t col_a(int set, int buf) { return kColA + 32u * (2 * set + buf); }
__host__ __device__ constexpr uint32_t col_d(int set, int buf) { return kColD + 16u * (2 * set + buf); }

template <int WBITS>
struct TcStage {
    static constexpr int kCB = WBITS == 4 ? 512 : 256;
    static constexpr int kWBytes = 2 * kGroupStrips * kCB;
    static constexpr int kXUnit = kRows * 128;  // 16 rows x 64 k x 2 B, 128B-swizzled
    static constexpr int kX = align_up(kWBytes, 1024);
    static constexpr int kS = kX + 2 * kXUnit;
    static constexpr int kBytes = align_up(kS + kGroupCols * 2, 1024);
    static constexpr int kRing = kStages * kBytes;
    static constexpr int kBars = 2 * kStages + 10;
    static constexpr int kSmem0 = 1024 + kRing + kBars * 8 + 16;
    static constexpr int kSmem = kSmem0 > kMinSmem ? kSmem0 : kMinSmem;
    // Split-K partials [2 sets][16 tokens][128 columns] fp32 reuse the ring.
    static_assert(2 * kRows * kGroupCols * 4 <= kRing, "partials fit in the ring");
};

struct alignas(64) DecodeTcParams {
    CUtensorMap x_map;  // [M][K] 16-bit activations: box 64 x 16, 128B swizzle, rows >= M read zero
    const uint8_t* W;
    const void* S;
    void* C;
    unsigned* err;
    int M, N, K, group;
    int cs;
    int early_weights;
};

template <bool kBF16>
__device__ __forceinline__ float scale_f32(uint16_t v) {
    if constexpr (kBF16) return __uint_as_float((uint32_t)v << 16);
    else return __half2float(__ushort_as_half(v));
}

// Four consecutive outputs (8- or 16-byte aligned: column offsets are multiples of 4).
template <typename OT>
__device__ __forceinline__ void store4(OT* dst, float4 v) {
    if constexpr (std::is_same<OT, float>::value) {
        *reinterpret_cast<float4*>(dst) = v;
    } else {
        OT h[4] = {from_f32<OT>(v.x), from_f32<OT>(v.y), from_f32<OT>(v.z), from_f32<OT>(v.w)};
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(h);
    }
}

// tcgen05.ld of 8 columns (tokens) of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

// kT = tokens drained per stage (8 when M <= 8, else 16).
template <int WBITS, typename AT, typename OT, int kT>
__global__ void __launch_bounds__(kThreads, 2) decode_tc_kernel(const __grid_constant__ DecodeTcParams p) {
    using L = TcStage<WBITS>;
    constexpr bool kBF16 = std::is_same<AT, __nv_bfloat16>::value;
    constexpr int kCB = L::kCB;
    constexpr uint32_t kIdesc = umma_idesc_f16(kBF16, 128, 16);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + L::kRing);
    uint64_t* empty = full + kStages;
    uint64_t* a_full = empty + kStages;  // [set][buf]: the four warps of the set
    uint64_t* d_full = a_full + 4;       // [set][buf]
    uint64_t* mma_done = d_full + 4;     // [set]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WBITS);
    const int KB = geo.KB;
    const int upg = p.group / kBlockK;  // k-blocks per scale group (even)
    const int G = KB / upg;
    const int cs = p.cs;
    const int sg = blockIdx.x / cs;
    const int rank = cs > 1 ? (int)cluster_ctarank() : 0;
    const int width = geo.width(sg);
    const int g_begin = rank * G / cs, g_end = (rank + 1) * G / cs;
    const int kb_begin = g_begin * upg;
    const int n_iters = (g_end - g_begin) * upg / 2;
    const uint32_t unit_bytes = (uint32_t)width * kCB;
    const size_t off0 = geo.unit_offset((long long)sg * KB + kb_begin);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 2);  // one commit per issuing thread
        }
        for (int i = 0; i < 4; ++i) mbar_init(&a_full[i], kDqWarps / 2);
        for (int i = 0; i < 4; ++i) mbar_init(&d_full[i], 1);
        for (int i = 0; i < 2; ++i) mbar_init(&mma_done[i], 1);
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        pdl_launch_dependents();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    float acc[kT];
#pragma unroll
    for (int i = 0; i < kT; ++i) acc[i] = 0.f;

    if (warp == kProducerWarp) {
        // ---------------------------------------------------------- producer
        const uint64_t pol = l2_policy_evict_first();
        const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
        const uint32_t s_bytes = (uint32_t)width * kStripCols * 2;
        auto issue_x = [&](int it) {
            uint8_t* st = ring + (it % kStages) * L::kBytes;
            if (lane == 0)
                for (int u = 0; u < 2; ++u)
                    tma_load_2d(st + L::kX + u * L::kXUnit, &p.x_map, (kb_begin + 2 * it + u) * kBlockK, 0,
                                &full[it % kStages]);
        };
        const int early = p.early_weights ? min(kStages, n_iters) : 0;
        if (!early) pdl_wait();
        int issued = 0;
        bool ok = true;
        for (int it = 0; it < n_iters; ++it) {
            const int slot = it % kStages;
            if (lane == 0 && ok) ok = mbar_wait(&empty[slot], ((uint32_t)(it / kStages) & 1u) ^ 1u, p.err);
            uint8_t* st = ring + slot * L::kBytes;
            if (lane == 0) {
                const uint32_t wbytes = 2 * unit_bytes;
                mbar_arrive_expect_tx(&full[slot], wbytes + 2 * (uint32_t)L::kXUnit + s_bytes);
                bulk_g2s_hint(st, p.W + off0 + (size_t)it * wbytes, wbytes, &full[slot], pol);
                const int gi = (kb_begin + 2 * it) / upg;
                bulk_g2s(st + L::kS, Sb + ((size_t)gi * p.N + (size_t)sg * kGroupCols) * 2, s_bytes, &full[slot]);
            }
            __syncwarp();
            if (it >= early) {
                issue_x(it);
            } else if (it == early - 1) {
                // The first stages' weights are in flight; wait for the previous
                // kernel (which may have written A), then add their activations.
                pdl_wait();
                for (int j = 0; j < early; ++j) issue_x(j);
            }
            issued = it + 1;
        }
        if (issued < early) {
            pdl_wait();
            for (int j = 0; j < issued; ++j) issue_x(j);
        }
        // Copies still in flight land before the ring is reused or the CTA exits.
        if (lane == 0)
            for (int it = issued - kStages < 0 ? 0 : issued - kStages; it < issued; ++it)
                mbar_wait(&full[it % kStages], (uint32_t)(it / kStages) & 1u, p.err);
        __syncwarp();
    } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
        // ------------------------------------------------------------- MMA
        // Warp 9 + u issues the MMAs of k-block u of every stage (set u's A).
        const int u = warp - kMmaWarp;
        if (lane == 0) {
            bool ok = true;
            for (int it = 0; it < n_iters; ++it) {
                const int slot = it % kStages, b = it & 1;
                // The set's four warps expanded this k-block (so the stage landed,
                // and the set's A and D buffers of stage it-2 are drained).
                if (ok) ok = mbar_wait(&a_full[2 * u + b], (uint32_t)(it >> 1) & 1u, p.err);
                tc_fence_after();
                const uint32_t xs = smem_u32(ring + slot * L::kBytes + L::kX + u * L::kXUnit);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    umma_ts_f16(tmem + col_d(u, b), tmem + col_a(u, b) + 8u * k, sw128_kmajor_desc(xs + 32 * k),
                                kIdesc, k != 0);
                umma_commit(&d_full[2 * u + b]);
                umma_commit(&empty[slot]);
            }
            umma_commit(&mma_done[u]);
            mbar_wait(&mma_done[u], 0u, p.err);
        }
        __syncwarp();
    } else {
        // --------------------------------------------------- dequant + drain
        const int set = warp >> 2, q = warp & 3;
        const int sl = 2 * q + (lane >> 4);  // strip of the group
        const int c = lane & 15, g = c & 7, hh = c >> 3;
        const int rot = WBITS == 4 ? (g >> 1) : ((g >> 2) + 2 * (lane >> 4));  // bank-conflict-free gather
        const bool valid = sl < width;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        float sc_prev = 0.f;
        bool ok = true;
        auto drain = [&](int i, float sc) {
            const int b = i & 1;
            if (ok) ok = mbar_wait(&d_full[2 * set + b], (uint32_t)(i >> 1) & 1u, p.err);
            __syncwarp();
            tc_fence_after();
            uint32_t v[8];
            tmem_ld8(tmem + lane_base + col_d(set, b), v);
            if constexpr (kT == 16) {
                uint32_t w[8];
                tmem_ld8(tmem + lane_base + col_d(set, b) + 8u, w);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[8 + j] = fmaf(__uint_as_float(w[j]), sc, acc[8 + j]);
            } else {
                tmem_ld_wait();
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(__uint_as_float(v[j]), sc, acc[j]);
        };
        for (int it = 0; it < n_iters; ++it) {
            const int slot = it % kStages, b = it & 1;
            if (ok) ok = mbar_wait(&full[slot], (uint32_t)(it / kStages) & 1u, p.err);
            __syncwarp();
            tc_fence_after();
            const uint8_t* st = ring + slot * L::kBytes;
            const uint8_t* wu = st + set * unit_bytes + sl * kCB;
            const float sc =
                valid ? scale_f32<kBF16>(*reinterpret_cast<const uint16_t*>(st + L::kS + 2 * (16 * sl + c))) : 0.f;
            const uint32_t ta = tmem + lane_base + col_a(set, b);
            uint32_t cw[WBITS == 4 ? 8 : 4];  // this column's codes, k order
            if constexpr (WBITS == 4) gather_column_u4(wu, g, hh, rot, valid, cw);
            else gather_column_t2(wu, g, hh, rot, valid, cw);
#pragma unroll
            for (int t = 0; t < 4; ++t) {  // tcgen05.st takes one warp-uniform column: k = 16t .. 16t+15
                uint32_t r[8];
                if constexpr (WBITS == 4) {
                    const uint2 w = make_uint2(cw[2 * t], cw[2 * t + 1]);
                    uint32_t lo[4], hi[4];
                    if constexpr (kBF16) {
                        dequant_u4_bf16(w.x, lo);
                        dequant_u4_bf16(w.y, hi);
                    } else {
                        dequant_u4_f16(w.x, lo);
                        dequant_u4_f16(w.y, hi);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        r[e] = lo[e];
                        r[4 + e] = hi[e];
                    }
                } else {
                    const uint32_t w = cw[t];
#pragma unroll
                    for (int e = 0; e < 8; ++e) r[e] = dequant_t2_pair<kBF16>(w, e);
                }
                tmem_st8(ta + 8u * t, r);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[2 * set + b]);
            if (it > 0) drain(it - 1, sc_prev);
            sc_prev = sc;
        }
        if (n_iters > 0) drain(n_iters - 1, sc_prev);
    }

    // ------------------------------------------------------------- epilogue
    // Partials [set][token][column] to this CTA's shared memory (the ring: every
    // copy has landed and every MMA that read it has completed), then C = the
    // sum over sets and over the cluster's CTAs, in a fixed order.
    float* red = reinterpret_cast<float*>(ring);
    tc_fence_before();
    __syncthreads();
    if (warp < kDqWarps) {
        const int set = warp >> 2, col = 32 * (warp & 3) + lane;
#pragma unroll
        for (int j = 0; j < kT; ++j) red[(set * kRows + j) * kGroupCols + col] = acc[j];
    }
    if (cs > 1) cluster_sync();
    else __syncthreads();
    OT* C = reinterpret_cast<OT*>(p.C);
    const int q4 = width * kStripCols / 4;  // float4 per token row
    const int total = p.M * q4;
    const int share = (total + cs - 1) / cs;
    const uint32_t red_s = smem_u32(red);
    for (int i = rank * share + (int)threadIdx.x; i < min(total, (rank + 1) * share); i += kThreads) {
        const int tok = i / q4, c4 = (i % q4) * 4;
        float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < cs; ++r) {
#pragma unroll
            for (int set = 0; set < 2; ++set) {
                const uint32_t a = red_s + 4u * (uint32_t)((set * kRows + tok) * kGroupCols + c4);
                const float4 v = cs > 1 ? ld_dsmem_f4(mapa_shared(a, (uint32_t)r))
                                        : *reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(red) +
                                                                           (a - red_s));
                s4.x += v.x;
                s4.y += v.y;
                s4.z += v.z;
                s4.w += v.w;
            }
        }
        store4(C + (size_t)tok * p.N + (size_t)sg * kGroupCols + c4, s4);
    }
    if (cs > 1) cluster_sync();
    else __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

using TcKernelFn = void (*)(DecodeTcParams);

struct TcKernelInfo {
    TcKernelFn fn = nullptr;
    int smem = 0;
};

template <int WBITS, typename AT, int kT>
TcKernelInfo tc_pick_out(DType c) {
    if (c == DType::F32) return {decode_tc_kernel<WBITS, AT, float, kT>, TcStage<WBITS>::kSmem};
    if (std::is_same<AT, __half>::value && c == DType::F16)
        return {decode_tc_kernel<WBITS, AT, AT, kT>, TcStage<WBITS>::kSmem};
    if (std::is_same<AT, __nv_bfloat16>::value && c == DType::BF16)
        return {decode_tc_kernel<WBITS, AT, AT, kT>, TcStage<WBITS>::kSmem};
    return {};
}

template <int kT>
TcKernelInfo tc_pick(const GemmArgs& a) {
    if (a.a_dtype == DType::F16)
        return a.wbits == 4 ? tc_pick_out<4, __half, kT>(a.c_dtype) : tc_pick_out<2, __half, kT>(a.c_dtype);
    if (a.a_dtype == DType::BF16)
        return a.wbits == 4 ? tc_pick_out<4, __nv_bfloat16, kT>(a.c_dtype)
                            : tc_pick_out<2, __nv_bfloat16, kT>(a.c_dtype);
    return {};
}

TcKernelInfo tc_select(const GemmArgs& a) {
    if (a.bias || a.group % 128 != 0 || a.M < 1 || a.M > kRows || a.s_dtype != a.a_dtype) return {};
    return a.M <= 8 ? tc_pick<8>(a) : tc_pick<16>(a);
}

// Clusters of cs CTAs resident at once (cached per function, cs and device).
int active_clusters(TcKernelFn fn, int smem, int cs, int dev) {
    static std::mutex mu;
    struct Entry {
        TcKernelFn fn;
        int cs, dev, val;
    };
    static Entry cache[128];
    static int n = 0;
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < n; ++i)
        if (cache[i].fn == fn && cache[i].cs == cs && cache[i].dev == dev) return cache[i].val;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(cs * 64));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int v = 0;
    if (cudaOccupancyMaxActiveClusters(&v, fn, &cfg) != cudaSuccess || v <= 0) {
        (void)cudaGetLastError();
        v = std::max(1, device_info(dev).sm_count * 2 / cs);
    }
    if (n < 128) cache[n++] = {fn, cs, dev, v};
    return v;
}

// CTAs per strip group: the cs in 1..8 (<= groups along K) minimising
// waves x groups per CTA, ties to the smaller cs (less reduction).
int tc_cluster_size(const TcKernelInfo& ki, int N, int K, int wbits, int group, int dev) {
    const TileGeom geo(K, N, wbits);
    const int G = K / group;
    int best = 1;
    long long best_cost = -1;
    for (int cs = 1; cs <= std::min(8, G); ++cs) {
        const long long clusters = active_clusters(ki.fn, ki.smem, cs, dev);
        const long long waves = (geo.NSG + clusters - 1) / clusters;
        const long long cost = waves * ((G + cs - 1) / cs) * 16 + cs;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = cs;
        }
    }
    return best;
}

}  // namespace

bool decode_tc_supported(const GemmArgs& a) { return tc_select(a).fn != nullptr; }

cudaError_t launch_decode_tc(const GemmArgs& a, bool early_weights) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const TcKernelInfo ki = tc_select(a);
    if (!ki.fn) return cudaErrorInvalidValue;
    e = ensure_smem_attr(reinterpret_cast<const void*>(ki.fn), dev, ki.smem);
    if (e != cudaSuccess) return e;
    const TileGeom geo(a.K, a.N, a.wbits);
    DecodeTcParams p;
    memset(&p, 0, sizeof p);
    e = make_tmap_2d(&p.x_map, a.A, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2,
                     kBlockK, kRows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    p.W = a.W;
    p.S = a.S;
    p.C = a.C;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.group = a.group;
    p.err = device_error_word(dev);
    p.cs = tc_cluster_size(ki, a.N, a.K, a.wbits, a.group, dev);
    p.early_weights = (early_weights && !a.weights_just_written) ? 1 : 0;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(geo.NSG * p.cs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)ki.smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, ki.fn, p);
}

}  // namespace hq
