// hq_decode.cu -- HBM-streaming W4A16 / ternary GEMM for decode (M <= 16).
//
// Replaces kernel_marlin_gemm_int4_templated / _dynamic and the memset +
// atomicAdd split-K of the reference (hydrogen/src/model/marlin_gemm.cu:130-322,
// :556-601).  Design for B200:
//   * Work = "units" (strip group of 128 columns, 64-k block).  The tile order
//     makes any run of consecutive units one contiguous byte span, so each
//     persistent CTA streams its unit range with large 1-D bulk copies (TMA
//     engine) into a multi-stage shared-memory ring -- one elected producer
//     thread, mbarrier full/empty handshakes, L2 evict-first hint.
//   * Four consumer warps each own two 16-column strips.  A lane's 16 bytes
//     are exactly its A fragments for four m16n8k16 steps: register dequant
//     (mask + OR into an fp16/bf16 exponent pattern, one packed subtract),
//     tensor-core MMA with fp32 accumulation, and the group scale applied to
//     each 64-k partial in fp32 (never rounded into the weight).
//   * Split-K across CTAs is deterministic: each CTA writes its partial for a
//     strip group to its own workspace slot; the last CTA to arrive (atomic
//     counter) sums the slots in CTA order and writes C, then resets the
//     counter to zero.  No memset, no float atomics, no spin-waits.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"

#include <algorithm>
#include <type_traits>

namespace hq {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kStripsPerWarp = 2;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageBytes = 8192;  // 2 int4 units / 4 ternary units of a full group
constexpr int kStages = 6;
constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8 + 16;

struct DecodeParams {
    const void* A;
    const uint8_t* W;
    const void* S;
    const float* bias;
    void* C;
    float* partials;     // [(P + NSG)][M][128]
    unsigned* counters;  // [NSG]
    unsigned* err;       // device error word
    int M, N, K, group;
    long long U;
};

// CTA that owns unit u when U units are split into P contiguous ranges
// [floor(U p / P), floor(U (p+1) / P)).
__device__ __forceinline__ int owner_of(long long u, long long U, int P) {
    return (int)(((u + 1) * (long long)P - 1) / U);
}

template <typename AT>
struct XFrag;

// fp16 / bf16 activations: two 16-byte loads hold the 16 k this lane needs.
template <typename AT>
struct XFrag {
    uint4 a, b;
    __device__ __forceinline__ void load(const AT* row, bool valid) {
        if (valid) {
            a = ldg128_nc(row);
            b = ldg128_nc(row + 8);
        } else {
            a = make_uint4(0, 0, 0, 0);
            b = a;
        }
    }
    __device__ __forceinline__ uint32_t b0(int step) const {
        return step == 0 ? a.x : step == 1 ? a.z : step == 2 ? b.x : b.z;
    }
    __device__ __forceinline__ uint32_t b1(int step) const {
        return step == 0 ? a.y : step == 1 ? a.w : step == 2 ? b.y : b.w;
    }
};

// fp32 activations: x = hi + lo with hi = fp16(x), lo = fp16(x - hi); two MMAs
// per step keep the product accurate to ~2^-22 relative.
struct XFragF32 {
    uint32_t hi[8], lo[8];
    __device__ __forceinline__ void load(const float* row, bool valid) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float4 v = valid ? *reinterpret_cast<const float4*>(row + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
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

template <typename AT>
struct ComputeType {
    static constexpr bool bf16 = false;
};
template <>
struct ComputeType<__nv_bfloat16> {
    static constexpr bool bf16 = true;
};

// A fragments (4 regs) of step `step` for this lane from its chunk words.
template <int WBITS, bool kBF16, bool kUnsigned>
struct WFrag {
    uint32_t r[4][4];  // [step][reg]
    __device__ __forceinline__ void build(uint4 w) {
        if constexpr (WBITS == 4) {
            uint32_t g0[4], g8[4];
            // words: x = row g k0..7, y = row g k8..15, z = row g+8 k0..7, w = row g+8 k8..15
            if constexpr (kBF16) {
                dequant_u4_bf16<kUnsigned>(w.x, g0);
                dequant_u4_bf16<kUnsigned>(w.z, g8);
            } else {
                dequant_u4_f16<kUnsigned>(w.x, g0);
                dequant_u4_f16<kUnsigned>(w.z, g8);
            }
            r[0][0] = g0[0]; r[0][1] = g8[0]; r[0][2] = g0[1]; r[0][3] = g8[1];
            r[1][0] = g0[2]; r[1][1] = g8[2]; r[1][2] = g0[3]; r[1][3] = g8[3];
            if constexpr (kBF16) {
                dequant_u4_bf16<kUnsigned>(w.y, g0);
                dequant_u4_bf16<kUnsigned>(w.w, g8);
            } else {
                dequant_u4_f16<kUnsigned>(w.y, g0);
                dequant_u4_f16<kUnsigned>(w.w, g8);
            }
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
__device__ __forceinline__ float load_scale(const void* S, size_t idx) {
    return to_f32(__ldg(reinterpret_cast<const ST*>(S) + idx));
}

template <int WBITS, int MT, typename AT, typename ST, typename OT, bool kBias>
__global__ void __launch_bounds__(kThreads) decode_kernel(const __grid_constant__ DecodeParams p) {
    constexpr bool kSplit = std::is_same<AT, float>::value;
    constexpr bool kBF16 = ComputeType<AT>::bf16;  // float activations compute in fp16
    constexpr int kCB = WBITS == 4 ? 512 : 256;
    constexpr int kLaneBytes = kCB / 32;

    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    int* s_flag = reinterpret_cast<int*>(empty + kStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WBITS);
    const int P = gridDim.x, pid = blockIdx.x;
    const long long u0 = p.U * pid / P, u1 = p.U * (pid + 1) / P;
    const int units_per_stage = kStageBytes / (kGroupStrips * kCB);
    const int n_iters = (int)((u1 - u0 + units_per_stage - 1) / units_per_stage);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;
            for (int it = 0; it < n_iters; ++it) {
                const int slot = it % kStages;
                const uint32_t ph = (uint32_t)(it / kStages) & 1u;
                if (!mbar_wait(&empty[slot], ph ^ 1u, p.err)) break;
                const long long ua = u0 + (long long)it * units_per_stage;
                const long long ub = ua + units_per_stage < u1 ? ua + units_per_stage : u1;
                const size_t oa = geo.unit_offset(ua);
                const uint32_t bytes = (uint32_t)(geo.unit_offset(ub) - oa);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_g2s_evict_first(ring + slot * kStageBytes, p.W + oa, bytes, &full[slot], pol);
                issued = it + 1;
            }
            // Copies still in flight land before this thread leaves.
            for (int it = issued - kStages < 0 ? 0 : issued - kStages; it < issued; ++it)
                mbar_wait(&full[it % kStages], (uint32_t)(it / kStages) & 1u, p.err);
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const int KB = geo.KB;
    float acc[kStripsPerWarp][MT][4];
#pragma unroll
    for (int j = 0; j < kStripsPerWarp; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][m][i] = 0.f;

    long long cur_sg = u0 / KB;

    auto flush = [&](long long sg) {
        const int width = geo.width((int)sg);
        const int f = owner_of(sg * KB, p.U, P);
        const int l = owner_of((sg + 1) * KB - 1, p.U, P);
        const int nc = l - f + 1;
        OT* C = reinterpret_cast<OT*>(p.C);
        if (nc == 1) {
#pragma unroll
            for (int j = 0; j < kStripsPerWarp; ++j) {
                const int sl = kStripsPerWarp * warp + j;
                if (sl >= width) continue;
                const int n = (int)(sg * kGroupCols) + sl * kStripCols + g;
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const int tok = 8 * m + 2 * t;
                    if (tok < p.M) {
                        C[(size_t)tok * p.N + n] = from_f32<OT>(acc[j][m][0]);
                        C[(size_t)tok * p.N + n + 8] = from_f32<OT>(acc[j][m][2]);
                    }
                    if (tok + 1 < p.M) {
                        C[(size_t)(tok + 1) * p.N + n] = from_f32<OT>(acc[j][m][1]);
                        C[(size_t)(tok + 1) * p.N + n + 8] = from_f32<OT>(acc[j][m][3]);
                    }
                }
            }
            return;
        }
        float* part = p.partials + (size_t)(pid + sg) * p.M * kGroupCols;
#pragma unroll
        for (int j = 0; j < kStripsPerWarp; ++j) {
            const int sl = kStripsPerWarp * warp + j;
            if (sl >= width) continue;
            const int nl = sl * kStripCols + g;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int tok = 8 * m + 2 * t;
                if (tok < p.M) {
                    part[tok * kGroupCols + nl] = acc[j][m][0];
                    part[tok * kGroupCols + nl + 8] = acc[j][m][2];
                }
                if (tok + 1 < p.M) {
                    part[(tok + 1) * kGroupCols + nl] = acc[j][m][1];
                    part[(tok + 1) * kGroupCols + nl + 8] = acc[j][m][3];
                }
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned old = atomicAdd(&p.counters[sg], 1u);
            *s_flag = (old == (unsigned)(nc - 1));
        }
        named_bar_sync(1, kConsumerWarps * 32);
        if (*s_flag) {
            __threadfence();
            const int cols = width * kStripCols;
            for (int e = threadIdx.x; e < p.M * kGroupCols; e += kConsumerWarps * 32) {
                const int tok = e / kGroupCols, nl = e % kGroupCols;
                if (nl >= cols) continue;
                float s = 0.f;
                for (int c = 0; c < nc; ++c)
                    s += __ldcg(p.partials + (size_t)(f + c + sg) * p.M * kGroupCols + e);
                C[(size_t)tok * p.N + sg * kGroupCols + nl] = from_f32<OT>(s);
            }
            if (threadIdx.x == 0) p.counters[sg] = 0u;
        }
    };

    const AT* A = reinterpret_cast<const AT*>(p.A);
    using XF = typename std::conditional<kSplit, XFragF32, XFrag<AT>>::type;
    const uint32_t kOnes = 0x3C003C00u;  // fp16 (1, 1) for the bias row sums

    // After a timed-out wait the warp stops waiting but keeps the same control
    // flow (results are garbage, the error word is set), so the named barriers
    // of the split-K flush always see all consumer warps: no hang either way.
    bool waits_ok = true;
    for (int it = 0; it < n_iters; ++it) {
        const int slot = it % kStages;
        if (waits_ok) waits_ok = mbar_wait(&full[slot], (uint32_t)(it / kStages) & 1u, p.err);
        const long long ua = u0 + (long long)it * units_per_stage;
        const long long ub = ua + units_per_stage < u1 ? ua + units_per_stage : u1;
        const size_t oa = geo.unit_offset(ua);
        const uint32_t stage_base = smem_u32(ring + slot * kStageBytes);
        for (long long u = ua; u < ub; ++u) {
            const long long sg = u / KB;
            const int kb = (int)(u % KB);
            if (sg != cur_sg) {
                flush(cur_sg);
#pragma unroll
                for (int j = 0; j < kStripsPerWarp; ++j)
#pragma unroll
                    for (int m = 0; m < MT; ++m)
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[j][m][i] = 0.f;
                cur_sg = sg;
            }
            const int width = geo.width((int)sg);
            const uint32_t unit_base = stage_base + (uint32_t)(geo.unit_offset(u) - oa);
            XF xf[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int tok = 8 * m + g;
                xf[m].load(A + (size_t)(tok < p.M ? tok : 0) * p.K + kb * kBlockK + 16 * t, tok < p.M);
            }
            const int gi = kb * kBlockK / p.group;
            // Row sums of x over this 64-k block (only for the bias form).
            float xs[MT][4];
            if constexpr (kBias) {
                const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
#pragma unroll
                for (int m = 0; m < MT; ++m) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) xs[m][i] = 0.f;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        if constexpr (kSplit) {
                            mma_16816<false>(xs[m], ones, xf[m].hi[2 * s], xf[m].hi[2 * s + 1]);
                            mma_16816<false>(xs[m], ones, xf[m].lo[2 * s], xf[m].lo[2 * s + 1]);
                        } else {
                            mma_16816<kBF16>(xs[m], ones, xf[m].b0(s), xf[m].b1(s));
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kStripsPerWarp; ++j) {
                const int sl = kStripsPerWarp * warp + j;
                if (sl >= width) continue;
                const uint32_t addr = unit_base + (uint32_t)(sl * kCB + lane * kLaneBytes);
                uint4 wv;
                if constexpr (WBITS == 4) {
                    wv = lds128(addr);
                } else {
                    uint2 v = lds64(addr);
                    wv = make_uint4(v.x, v.y, 0, 0);
                }
                const int n = (int)(sg * kGroupCols) + sl * kStripCols + g;
                const size_t si = (size_t)gi * p.N + n;
                float sc0, sc1;
                if constexpr (std::is_same<ST, float>::value) {
                    sc0 = __ldg(reinterpret_cast<const float*>(p.S) + si);
                    sc1 = __ldg(reinterpret_cast<const float*>(p.S) + si + 8);
                } else {
                    sc0 = load_scale<ST>(p.S, si);
                    sc1 = load_scale<ST>(p.S, si + 8);
                }
                WFrag<WBITS, kBF16, kBias> wf;
                wf.build(wv);
                float tmp[MT][4];
#pragma unroll
                for (int m = 0; m < MT; ++m) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) tmp[m][i] = 0.f;
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        if constexpr (kSplit) {
                            mma_16816<false>(tmp[m], wf.r[s], xf[m].hi[2 * s], xf[m].hi[2 * s + 1]);
                            mma_16816<false>(tmp[m], wf.r[s], xf[m].lo[2 * s], xf[m].lo[2 * s + 1]);
                        } else {
                            mma_16816<kBF16>(tmp[m], wf.r[s], xf[m].b0(s), xf[m].b1(s));
                        }
                    }
                }
                if constexpr (kBias) {
                    const float b0 = __ldg(p.bias + si), b1 = __ldg(p.bias + si + 8);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        acc[j][m][0] += tmp[m][0] * sc0 + xs[m][0] * b0;
                        acc[j][m][1] += tmp[m][1] * sc0 + xs[m][1] * b0;
                        acc[j][m][2] += tmp[m][2] * sc1 + xs[m][2] * b1;
                        acc[j][m][3] += tmp[m][3] * sc1 + xs[m][3] * b1;
                    }
                } else {
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        acc[j][m][0] = fmaf(tmp[m][0], sc0, acc[j][m][0]);
                        acc[j][m][1] = fmaf(tmp[m][1], sc0, acc[j][m][1]);
                        acc[j][m][2] = fmaf(tmp[m][2], sc1, acc[j][m][2]);
                        acc[j][m][3] = fmaf(tmp[m][3], sc1, acc[j][m][3]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (n_iters > 0) flush(cur_sg);
}

using KernelFn = void (*)(DecodeParams);

template <int WBITS, int MT, typename AT, typename ST, typename OT, bool kBias>
KernelFn kernel_ptr() {
    return decode_kernel<WBITS, MT, AT, ST, OT, kBias>;
}

// Output dtype: the activation's own 16-bit type or f32 (f32 activations: f32 out).
template <int WBITS, int MT, typename AT, typename ST, bool kBias>
KernelFn pick_out(DType c) {
    if (c == DType::F32) return kernel_ptr<WBITS, MT, AT, ST, float, kBias>();
    if constexpr (std::is_same<AT, __half>::value) {
        if (c == DType::F16) return kernel_ptr<WBITS, MT, AT, ST, __half, kBias>();
    }
    if constexpr (std::is_same<AT, __nv_bfloat16>::value) {
        if (c == DType::BF16) return kernel_ptr<WBITS, MT, AT, ST, __nv_bfloat16, kBias>();
    }
    return nullptr;
}

// Supported (activation, scale, bias) combinations.  int4: (f16,f16), (bf16,bf16),
// (f16|bf16, f32), (f32, f32) with or without bias for f16/f32 activations, and
// (f32, f16).  Ternary: (f16,f16), (bf16,bf16).
template <int WBITS, int MT>
KernelFn pick(const GemmArgs& a) {
    const bool bias = a.bias != nullptr;
    if (a.a_dtype == DType::F16 && a.s_dtype == DType::F16 && !bias)
        return pick_out<WBITS, MT, __half, __half, false>(a.c_dtype);
    if (a.a_dtype == DType::BF16 && a.s_dtype == DType::BF16 && !bias)
        return pick_out<WBITS, MT, __nv_bfloat16, __nv_bfloat16, false>(a.c_dtype);
    if constexpr (WBITS == 4) {
        if (a.a_dtype == DType::F16 && a.s_dtype == DType::F32)
            return bias ? pick_out<WBITS, MT, __half, float, true>(a.c_dtype)
                        : pick_out<WBITS, MT, __half, float, false>(a.c_dtype);
        if (a.a_dtype == DType::BF16 && a.s_dtype == DType::F32 && !bias)
            return pick_out<WBITS, MT, __nv_bfloat16, float, false>(a.c_dtype);
        if (a.a_dtype == DType::F32 && a.s_dtype == DType::F32)
            return bias ? pick_out<WBITS, MT, float, float, true>(a.c_dtype)
                        : pick_out<WBITS, MT, float, float, false>(a.c_dtype);
        if (a.a_dtype == DType::F32 && a.s_dtype == DType::F16 && !bias)
            return pick_out<WBITS, MT, float, __half, false>(a.c_dtype);
    }
    return nullptr;
}

KernelFn select_kernel(const GemmArgs& a) {
    const int MT = a.M <= 8 ? 1 : 2;
    if (a.wbits == 4) return MT == 1 ? pick<4, 1>(a) : pick<4, 2>(a);
    return MT == 1 ? pick<2, 1>(a) : pick<2, 2>(a);
}

int grid_size(int M, long long U, int dev) {
    const DeviceInfo& di = device_info(dev);
    // Resident CTAs per SM is bounded by shared memory (48 KB ring each);
    // decode_workspace_bytes relies on this bound (sm_count * 4).
    const int per_sm = 4;
    long long P = (long long)di.sm_count * per_sm;
    // Larger M makes each split-K partial dearer; keep >= min_units per CTA.
    const long long min_units = M <= 8 ? 4 : 8;
    P = std::min(P, std::max<long long>(1, U / min_units));
    P = std::min(P, U);
    return (int)std::max<long long>(P, 1);
}

}  // namespace

bool decode_supported(const GemmArgs& a) { return select_kernel(a) != nullptr; }

size_t decode_workspace_bytes(int M, int N, int K, int wbits, int dev) {
    const TileGeom geo(K, N, wbits);
    // Slot count bound for any launch with <= M rows: grid_size() never exceeds
    // sm_count * 4, and a launch uses (grid + groups) slots of (rows x 128) floats.
    const long long P = (long long)device_info(dev).sm_count * 4;
    size_t part = (size_t)(P + geo.NSG) * (size_t)M * kGroupCols * sizeof(float);
    size_t cnt = (size_t)geo.NSG * sizeof(unsigned);
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    return up(cnt) + up(part);
}

cudaError_t launch_decode(const GemmArgs& a) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const TileGeom geo(a.K, a.N, a.wbits);
    KernelFn fn = select_kernel(a);
    if (!fn) return cudaErrorInvalidValue;
    e = ensure_smem_attr(reinterpret_cast<const void*>(fn), dev, kSmemBytes);
    if (e != cudaSuccess) return e;
    DecodeParams p;
    p.A = a.A;
    p.W = a.W;
    p.S = a.S;
    p.bias = a.bias;
    p.C = a.C;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.group = a.group;
    p.U = geo.units();
    p.err = device_error_word(dev);
    const int P = grid_size(a.M, p.U, dev);
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    p.counters = reinterpret_cast<unsigned*>(a.ws);
    p.partials = reinterpret_cast<float*>(a.ws + up((size_t)geo.NSG * sizeof(unsigned)));
    fn<<<P, kThreads, kSmemBytes, a.stream>>>(p);
    return cudaGetLastError();
}

}  // namespace hq
