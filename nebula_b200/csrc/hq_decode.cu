// hq_decode.cu -- HBM-streaming W4A16 / ternary GEMM for decode (M <= 16).
//
// Replaces kernel_marlin_gemm_int4_templated / _dynamic and the memset +
// atomicAdd split-K of the reference (hydrogen/src/model/marlin_gemm.cu:130-322,
// :556-601).  Design for B200:
//   * Work = strip groups of 128 output columns.  A thread-block cluster of cs
//     CTAs (cs in {1,2,4,8,10,12}, chosen from the measured cluster occupancy
//     so the grid fills the GPU) owns one strip
//     group; CTA r of the cluster streams the group's k-blocks
//     [r KB/cs, (r+1) KB/cs), which the tile order stores as one contiguous
//     byte span.  One producer warp moves it with 1-D bulk copies (TMA engine)
//     into a 4-stage shared-memory ring, two 64-k blocks per stage, together
//     with each block's activation tile (one 2-D TMA box of 16 rows x 64 k,
//     128-byte swizzled, rows >= M zero-filled) and group-scale row, so the
//     consumer loop reads only shared memory.  L2 evict-first on the weights.
//   * Four consumer warps each own two 16-column strips.  A lane's 16 bytes
//     are its A fragments for four m16n8k16 steps: codes are OR-ed into an
//     fp16/bf16 exponent pattern (one LOP3 per pair) and fed to the tensor
//     cores; one packed subtract per pair gives exact q.  fp32
//     accumulation; the group scale is applied in fp32 once per group within a
//     stage (never rounded into the weight).
//   * Split-K reduction through distributed shared memory: each CTA leaves its
//     fp32 partial in its own shared memory, and after a cluster barrier CTA r
//     sums 1/cs of the tile over the cs CTAs in rank order (deterministic) and
//     writes C.  No workspace, no atomics, no memset.
//   * Programmatic dependent launch: each CTA lets the next kernel on the
//     stream start immediately; weights and scales (which no earlier kernel
//     writes) are requested before griddepcontrol.wait, activations after it,
//     so the next GEMM's weight stream overlaps this GEMM's tail.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"
#include "hq_tmap.h"

#include <algorithm>
#include <cstring>
#include <type_traits>

namespace hq {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kStripsPerWarp = 2;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kUPS = 2;  // 64-k blocks per stage
constexpr int kMaxRows = 16;

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// Shared-memory layout of one pipeline stage.  kG32: scale groups of 32 k, so
// each 64-k block has two scale (and bias) rows.
template <int WBITS, typename AT, typename ST, bool kBias, bool kG32, int kNStages = 4>
struct Stage {
    static constexpr int kCB = WBITS == 4 ? 512 : 256;
    static constexpr int kWBytes = kUPS * kGroupStrips * kCB;  // weights of a full group
    static constexpr bool kXTma = sizeof(AT) == 2;            // 16-bit activations: one TMA box per block
    static constexpr int kXElt = (int)sizeof(AT);
    static constexpr int kXRowBytes = kBlockK * kXElt;             // activation bytes per row and block
    static constexpr int kXRow = kXTma ? 128 : kXRowBytes + 16;   // 128B-swizzled rows / padded rows
    static constexpr int kXUnit = kMaxRows * kXRow;
    static constexpr int kSElt = (int)sizeof(ST);
    static constexpr int kSRows = kG32 ? 2 : 1;  // scale rows per k-block
    static constexpr int kSRow = kGroupCols * kSElt;
    static constexpr int kSUnit = kSRows * kSRow;
    static constexpr int kBRow = kGroupCols * 4;
    static constexpr int kBUnit = kBias ? kSRows * kBRow : 0;
    static constexpr int kX = align_up(kWBytes, 1024);  // swizzled TMA destination: 1024-byte aligned
    static constexpr int kS = kX + kUPS * kXUnit;
    static constexpr int kB = kS + kUPS * kSUnit;
    static constexpr int kBytes = align_up(kB + kUPS * kBUnit, 1024);
    static constexpr int kStages = kNStages;
    static constexpr int kSmem = kStages * kBytes + 1024 /* base alignment slack */ + 2 * kStages * 8;
};

struct alignas(64) DecodeParams {
    CUtensorMap x_map;  // 16-bit activations [M][K]: box 64 x 16, 128B swizzle, OOB rows read zero
    const void* A;
    const uint8_t* W;
    const void* S;
    const float* bias;
    void* C;
    unsigned* err;  // device error word
    int M, N, K, group;
    int cs;             // CTAs per strip group (cluster size)
    int early_weights;  // stream weights/scales before the previous kernel finishes
};

// fp16 / bf16 activations: the 16 k (4 MMA steps) of one token row for this lane.
template <typename AT>
struct XFrag {
    uint4 a, b;
    // TMA tile: row `r`, 16-byte chunks c at ((c ^ (r & 7)) << 4) (128B swizzle).
    __device__ __forceinline__ void load(const uint8_t* tile, int r, int t) {
        const uint8_t* row = tile + r * 128;
        a = *reinterpret_cast<const uint4*>(row + (((2 * t) ^ (r & 7)) << 4));
        b = *reinterpret_cast<const uint4*>(row + (((2 * t + 1) ^ (r & 7)) << 4));
    }
    // TILE_U4_K32 order: lane t takes chunks t (k 8t..) and t + 4 (k 32 + 8t..).  Odd
    // rows read the upper chunk first, so the 8 lanes of each quarter warp (rows
    // 2i, 2i + 1) hit 8 different chunk slots on either load.
    __device__ __forceinline__ void load_k32(const uint8_t* tile, int r, int t) {
        const uint8_t* row = tile + r * 128;
        const bool odd = r & 1;
        const uint4 p = *reinterpret_cast<const uint4*>(row + (((odd ? t + 4 : t) ^ (r & 7)) << 4));
        const uint4 q = *reinterpret_cast<const uint4*>(row + (((odd ? t : t + 4) ^ (r & 7)) << 4));
        a = odd ? q : p;
        b = odd ? p : q;
    }
    __device__ __forceinline__ uint32_t b0(int step) const {
        return step == 0 ? a.x : step == 1 ? a.z : step == 2 ? b.x : b.z;
    }
    __device__ __forceinline__ uint32_t b1(int step) const {
        return step == 0 ? a.y : step == 1 ? a.w : step == 2 ? b.y : b.w;
    }
};

// fp32 activations (padded rows): x = hi + lo with hi = fp16(x), lo = fp16(x - hi);
// two MMAs per step keep the product accurate to ~2^-22 relative.
struct XFragF32 {
    uint32_t hi[8], lo[8];
    // k32: TILE_U4_K32 order, floats 8t.. (steps 0, 1) and 32 + 8t.. (steps 2, 3).
    __device__ __forceinline__ void load(const uint8_t* tile, int r, int t, bool k32 = false) {
        const uint8_t* row = tile + r * (kBlockK * 4 + 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint8_t* sp = k32 ? row + 32 * t + 128 * (i >> 1) + 16 * (i & 1) : row + 64 * t + 16 * i;
            uint4 q = *reinterpret_cast<const uint4*>(sp);
            float4 v = make_float4(__uint_as_float(q.x), __uint_as_float(q.y), __uint_as_float(q.z),
                                   __uint_as_float(q.w));
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

// A fragments (4 regs) of each of the four m16n8k16 steps from a lane's chunk words.
// kRaw: raw "magic + code" values (see hq_common.cuh); otherwise exact q (or u).
template <int WBITS, bool kBF16, bool kUnsigned, bool kRaw>
struct WFrag {
    uint32_t r[4][4];  // [step][reg]
    __device__ __forceinline__ void expand(uint32_t w, uint32_t (&o)[4]) {
        if constexpr (kRaw) {
            if constexpr (kBF16)
                raw_u4_bf16(w, o);
            else
                raw_u4_f16(w, o);
        } else {
            if constexpr (kBF16)
                dequant_u4_bf16<kUnsigned>(w, o);
            else
                dequant_u4_f16<kUnsigned>(w, o);
        }
    }
    __device__ __forceinline__ void build(uint4 w) {
        if constexpr (WBITS == 4) {
            uint32_t g0[4], g8[4];
            // words: x = row g k0..7, y = row g k8..15, z = row g+8 k0..7, w = row g+8 k8..15
            expand(w.x, g0);
            expand(w.z, g8);
            r[0][0] = g0[0]; r[0][1] = g8[0]; r[0][2] = g0[1]; r[0][3] = g8[1];
            r[1][0] = g0[2]; r[1][1] = g8[2]; r[1][2] = g0[3]; r[1][3] = g8[3];
            expand(w.y, g0);
            expand(w.w, g8);
            r[2][0] = g0[0]; r[2][1] = g8[0]; r[2][2] = g0[1]; r[2][3] = g8[1];
            r[3][0] = g0[2]; r[3][1] = g8[2]; r[3][2] = g0[3]; r[3][3] = g8[3];
        } else {
            // words: x = row g k0..15, y = row g+8 k0..15
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                if constexpr (kRaw) {
                    r[s][0] = raw_t2_pair<kBF16>(w.x, 2 * s);
                    r[s][1] = raw_t2_pair<kBF16>(w.y, 2 * s);
                    r[s][2] = raw_t2_pair<kBF16>(w.x, 2 * s + 1);
                    r[s][3] = raw_t2_pair<kBF16>(w.y, 2 * s + 1);
                } else {
                    r[s][0] = dequant_t2_pair<kBF16>(w.x, 2 * s);
                    r[s][1] = dequant_t2_pair<kBF16>(w.y, 2 * s);
                    r[s][2] = dequant_t2_pair<kBF16>(w.x, 2 * s + 1);
                    r[s][3] = dequant_t2_pair<kBF16>(w.y, 2 * s + 1);
                }
            }
        }
    }
};

// Raw-value correction: the A constant whose MMA with step s's activation
// fragment gives -(M + offset) * sum(x) (fp16 int4: odd steps see x/16 and
// weights 1024 + 16u, hence 1152 = 72 * 16).
template <int WBITS, bool kBF16>
__device__ __forceinline__ uint32_t raw_corr_const(int step) {
    if constexpr (WBITS == 4) {
        if constexpr (kBF16) return 0xC308C308u;                   // -136
        else return (step & 1) ? 0xE480E480u : 0xE408E408u;       // -1152 / -1032
    } else {
        return kBF16 ? 0xC301C301u : 0xE401E401u;                  // -129 / -1025
    }
}

template <typename ST>
__device__ __forceinline__ float lds_scale(const uint8_t* sp) {
    return to_f32(*reinterpret_cast<const ST*>(sp));
}

template <int WBITS, int MT, typename AT, typename ST, typename OT, bool kBias, bool kG32, int kNStages = 4>
__global__ void __launch_bounds__(kThreads, MT == 1 ? 4 : 3) decode_kernel(const __grid_constant__ DecodeParams p) {
    using L = Stage<WBITS, AT, ST, kBias, kG32, kNStages>;
    constexpr bool kSplit = std::is_same<AT, float>::value;
    constexpr bool kBF16 = ComputeType<AT>::bf16;  // float activations compute in fp16
    constexpr int kCB = L::kCB;
    constexpr int kLaneBytes = kCB / 32;
    constexpr int kStages = L::kStages;
    // Raw path (M <= 8 with fp16/bf16 activations, symmetric weights): MMA on
    // magic + code, offset removed by the per-block correction that seeds the
    // accumulator.  M > 8 subtracts on the FMA pipe instead, sparing the
    // legacy MMA rate which binds there.
    constexpr bool kRaw = false;
    constexpr bool kHiScale = kRaw && WBITS == 4 && !kBF16;  // fp16 int4: x/16 on odd steps

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * L::kBytes);
    uint64_t* empty = full + kStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WBITS);
    const int KB = geo.KB;
    const int cs = p.cs;
    const int sg = blockIdx.x / cs;
    const int rank = cs > 1 ? (int)cluster_ctarank() : 0;
    const int width = geo.width(sg);
    const int kb_begin = rank * KB / cs, kb_end = (rank + 1) * KB / cs;
    const int n_units = kb_end - kb_begin;
    const int n_iters = (n_units + kUPS - 1) / kUPS;
    const uint32_t unit_bytes = (uint32_t)width * kCB;  // one k-block of this strip group
    const size_t off0 = geo.unit_offset((long long)sg * KB + kb_begin);
    const int upg = kG32 ? 1 : p.group / kBlockK;  // k-blocks per scale group (group >= 64)

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kConsumerWarps);
        }
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        pdl_launch_dependents();
    }
    __syncthreads();

    float acc[kStripsPerWarp][MT][4];
#pragma unroll
    for (int j = 0; j < kStripsPerWarp; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][m][i] = 0.f;

    if (warp == kConsumerWarps) {
        // ---------------------------------------------------------- producer
        const uint64_t pol = l2_policy_evict_first();
        const uint8_t* Ab = reinterpret_cast<const uint8_t*>(p.A);
        const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
        const uint8_t* Bb = reinterpret_cast<const uint8_t*>(p.bias);
        const uint32_t cols = (uint32_t)width * kStripCols;
        const uint32_t s_bytes = cols * L::kSElt, b_bytes = kBias ? cols * 4 : 0;
        const uint32_t x_bytes = L::kXTma ? (uint32_t)L::kXUnit : (uint32_t)(p.M * L::kXRowBytes);
        // Activation tiles of stage `it` (the part that depends on the previous kernel).
        auto issue_x = [&](int it) {
            const int slot = it % kStages;
            uint8_t* st = ring + slot * L::kBytes;
            const int nu = min(kUPS, n_units - it * kUPS);
            if constexpr (L::kXTma) {
                if (lane == 0)
                    for (int ul = 0; ul < nu; ++ul)
                        tma_load_2d(st + L::kX + ul * L::kXUnit, &p.x_map, (kb_begin + it * kUPS + ul) * kBlockK, 0,
                                    &full[slot]);
            } else {
#pragma unroll
                for (int ul = 0; ul < kUPS; ++ul) {
                    if (ul < nu && lane < p.M) {
                        const int kb = kb_begin + it * kUPS + ul;
                        bulk_g2s(st + L::kX + ul * L::kXUnit + lane * L::kXRow,
                                 Ab + ((size_t)lane * p.K + (size_t)kb * kBlockK) * L::kXElt, L::kXRowBytes,
                                 &full[slot]);
                    }
                }
            }
        };
        const int early = p.early_weights ? min(kStages, n_iters) : 0;
        if (!early) pdl_wait();
        int issued = 0;
        for (int it = 0; it < n_iters; ++it) {
            const int slot = it % kStages;
            const uint32_t ph = (uint32_t)(it / kStages) & 1u;
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&empty[slot], ph ^ 1u, p.err);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const int nu = min(kUPS, n_units - it * kUPS);
            uint8_t* st = ring + slot * L::kBytes;
            if (lane == 0) {
                const uint32_t wbytes = (uint32_t)nu * unit_bytes;
                mbar_arrive_expect_tx(&full[slot],
                                      wbytes + (uint32_t)nu * (x_bytes + L::kSRows * (s_bytes + b_bytes)));
                bulk_g2s_hint(st, p.W + off0 + (size_t)it * kUPS * unit_bytes, wbytes, &full[slot], pol);
            }
            __syncwarp();
            // scale (and bias) rows of each k-block: [group][the 128 columns]
            if (lane >= 16 && lane < 16 + nu) {
                const int i = lane - 16;
                const int kb = kb_begin + it * kUPS + i;
#pragma unroll
                for (int h = 0; h < L::kSRows; ++h) {
                    const int gi = kG32 ? 2 * kb + h : kb / upg;
                    const size_t off = (size_t)gi * p.N + (size_t)sg * kGroupCols;
                    bulk_g2s(st + L::kS + i * L::kSUnit + h * L::kSRow, Sb + off * L::kSElt, s_bytes, &full[slot]);
                    if constexpr (kBias)
                        bulk_g2s(st + L::kB + i * L::kBUnit + h * L::kBRow, Bb + off * 4, b_bytes, &full[slot]);
                }
            }
            if (it >= early) {
                issue_x(it);
            } else if (it == early - 1) {
                // First stages' weights are in flight; now wait for the previous
                // kernel (which may have produced A) and add their activations.
                pdl_wait();
                for (int j = 0; j < early; ++j) issue_x(j);
            }
            issued = it + 1;
        }
        if (issued < early) {  // timed out before the early stages were completed
            pdl_wait();
            for (int j = 0; j < issued; ++j) issue_x(j);
        }
        // Copies still in flight land before the ring is reused or the CTA exits.
        if (lane == 0)
            for (int it = issued - kStages < 0 ? 0 : issued - kStages; it < issued; ++it)
                mbar_wait(&full[it % kStages], (uint32_t)(it / kStages) & 1u, p.err);
        __syncwarp();
    } else {
        // -------------------------------------------------------- consumers
        const int g = lane >> 2, t = lane & 3;
        using XF = typename std::conditional<kSplit, XFragF32, XFrag<AT>>::type;
        const uint32_t kOnes = 0x3C003C00u;  // fp16 (1, 1) for the bias row sums
        // Group 32 (TILE_U4_K32 weights): MMA steps 0, 1 of a block cover its
        // k [0, 32) (scale group 2kb), steps 2, 3 its k [32, 64) (group 2kb + 1).
        constexpr int kStepsPerRow = kG32 ? 2 : 4;  // MMA steps per scale row
        // After a timed-out wait the warp stops waiting but keeps the same
        // control flow (results are garbage, the error word is set): every
        // thread still reaches the barriers below, so nothing hangs.
        bool waits_ok = true;
        for (int it = 0; it < n_iters; ++it) {
            const int slot = it % kStages;
            if (waits_ok) waits_ok = mbar_wait(&full[slot], (uint32_t)(it / kStages) & 1u, p.err);
            const int nu = min(kUPS, n_units - it * kUPS);
            const int kb0 = kb_begin + it * kUPS;
            // Both blocks of the stage in one scale group: one scale application.
            const bool same = nu == 2 && (kb0 % upg) != upg - 1;
            const uint8_t* stage = ring + slot * L::kBytes;

            // Activation fragments (and raw-path corrections) of the stage's blocks.
            XF xf[kUPS][MT];
            float corr[kUPS][MT][4];
            // Activation sums for the bias term, per token: the ones-MMA gives rows
            // g and g + 8 the same value, so only its c0 / c1 are kept.
            float xs[kUPS][L::kSRows][MT][2];
#pragma unroll
            for (int u = 0; u < kUPS; ++u) {
                if (u >= nu) continue;
                const uint8_t* tile = stage + L::kX + u * L::kXUnit;
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if constexpr (!kG32) xf[u][m].load(tile, 8 * m + g, t);
                    else if constexpr (kSplit) xf[u][m].load(tile, 8 * m + g, t, true);
                    else xf[u][m].load_k32(tile, 8 * m + g, t);
                }
                // Rows >= M are zero (TMA fill) or stale (padded copies); either way
                // they only feed MMA columns (tokens) that are never stored.
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int i = 0; i < 4; ++i) corr[u][m][i] = 0.f;
                if constexpr (kRaw) {
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if constexpr (kHiScale) {
                            const uint32_t kSixteenth = 0x2C002C00u;
                            xf[u][m].a.z = hmul2_bits(xf[u][m].a.z, kSixteenth);
                            xf[u][m].a.w = hmul2_bits(xf[u][m].a.w, kSixteenth);
                            xf[u][m].b.z = hmul2_bits(xf[u][m].b.z, kSixteenth);
                            xf[u][m].b.w = hmul2_bits(xf[u][m].b.w, kSixteenth);
                        }
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            const uint32_t c = raw_corr_const<WBITS, kBF16>(s);
                            const uint32_t ca[4] = {c, c, c, c};
                            mma_16816<kBF16>(corr[u][m], ca, xf[u][m].b0(s), xf[u][m].b1(s));
                        }
                    }
                }
                if constexpr (kBias) {
                    const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
#pragma unroll
                    for (int h = 0; h < L::kSRows; ++h) {
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            float x4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int s = kStepsPerRow * h; s < kStepsPerRow * (h + 1); ++s) {
                                if constexpr (kSplit) {
                                    mma_16816<false>(x4, ones, xf[u][m].hi[2 * s], xf[u][m].hi[2 * s + 1]);
                                    mma_16816<false>(x4, ones, xf[u][m].lo[2 * s], xf[u][m].lo[2 * s + 1]);
                                } else {
                                    mma_16816<kBF16>(x4, ones, xf[u][m].b0(s), xf[u][m].b1(s));
                                }
                            }
                            xs[u][h][m][0] = x4[0];
                            xs[u][h][m][1] = x4[1];
                        }
                    }
                }
            }

#pragma unroll
            for (int j = 0; j < kStripsPerWarp; ++j) {
                const int sl = kStripsPerWarp * warp + j;
                if (sl >= width) continue;
                const int nl = sl * kStripCols + g;
                if constexpr (kG32) {
#pragma unroll
                    for (int u = 0; u < kUPS; ++u) {
                        if (u >= nu) continue;
                        const uint4 wv =
                            *reinterpret_cast<const uint4*>(stage + u * unit_bytes + sl * kCB + lane * kLaneBytes);
                        WFrag<WBITS, kBF16, kBias, false> wf;
                        wf.build(wv);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float tacc[MT][4];
#pragma unroll
                            for (int m = 0; m < MT; ++m) {
#pragma unroll
                                for (int i = 0; i < 4; ++i) tacc[m][i] = 0.f;
#pragma unroll
                                for (int s = 2 * h; s < 2 * h + 2; ++s) {
                                    if constexpr (kSplit) {
                                        mma_16816<false>(tacc[m], wf.r[s], xf[u][m].hi[2 * s], xf[u][m].hi[2 * s + 1]);
                                        mma_16816<false>(tacc[m], wf.r[s], xf[u][m].lo[2 * s], xf[u][m].lo[2 * s + 1]);
                                    } else {
                                        mma_16816<kBF16>(tacc[m], wf.r[s], xf[u][m].b0(s), xf[u][m].b1(s));
                                    }
                                }
                            }
                            const uint8_t* sp = stage + L::kS + u * L::kSUnit + h * L::kSRow;
                            const float s0 = lds_scale<ST>(sp + nl * L::kSElt);
                            const float s1 = lds_scale<ST>(sp + (nl + 8) * L::kSElt);
                            if constexpr (kBias) {
                                const uint8_t* bp = stage + L::kB + u * L::kBUnit + h * L::kBRow;
                                const float b0 = lds_scale<float>(bp + nl * 4), b1 = lds_scale<float>(bp + (nl + 8) * 4);
#pragma unroll
                                for (int m = 0; m < MT; ++m) {
                                    acc[j][m][0] += tacc[m][0] * s0 + xs[u][h][m][0] * b0;
                                    acc[j][m][1] += tacc[m][1] * s0 + xs[u][h][m][1] * b0;
                                    acc[j][m][2] += tacc[m][2] * s1 + xs[u][h][m][0] * b1;
                                    acc[j][m][3] += tacc[m][3] * s1 + xs[u][h][m][1] * b1;
                                }
                            } else {
#pragma unroll
                                for (int m = 0; m < MT; ++m) {
                                    acc[j][m][0] = fmaf(tacc[m][0], s0, acc[j][m][0]);
                                    acc[j][m][1] = fmaf(tacc[m][1], s0, acc[j][m][1]);
                                    acc[j][m][2] = fmaf(tacc[m][2], s1, acc[j][m][2]);
                                    acc[j][m][3] = fmaf(tacc[m][3], s1, acc[j][m][3]);
                                }
                            }
                        }
                    }
                    continue;
                }
                float tacc[kUPS][MT][4];  // per-block partial sums (independent MMA chains)
#pragma unroll
                for (int u = 0; u < kUPS; ++u) {
                    if (u >= nu) continue;
                    const uint8_t* wp = stage + u * unit_bytes + sl * kCB + lane * kLaneBytes;
                    uint4 wv;
                    if constexpr (WBITS == 4) {
                        wv = *reinterpret_cast<const uint4*>(wp);
                    } else {
                        const uint2 v = *reinterpret_cast<const uint2*>(wp);
                        wv = make_uint4(v.x, v.y, 0, 0);
                    }
                    WFrag<WBITS, kBF16, kBias, kRaw> wf;
                    wf.build(wv);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if constexpr (kSplit) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) tacc[u][m][i] = 0.f;
#pragma unroll
                            for (int s = 0; s < 4; ++s) {
                                mma_16816<false>(tacc[u][m], wf.r[s], xf[u][m].hi[2 * s], xf[u][m].hi[2 * s + 1]);
                                mma_16816<false>(tacc[u][m], wf.r[s], xf[u][m].lo[2 * s], xf[u][m].lo[2 * s + 1]);
                            }
                        } else {
                            mma_16816_c<kBF16>(tacc[u][m], wf.r[0], xf[u][m].b0(0), xf[u][m].b1(0), corr[u][m]);
#pragma unroll
                            for (int s = 1; s < 4; ++s)
                                mma_16816<kBF16>(tacc[u][m], wf.r[s], xf[u][m].b0(s), xf[u][m].b1(s));
                        }
                    }
                }
                // Apply the group scales (and the bias term of the reference form).
                const uint8_t* s0p = stage + L::kS;
                const float sa0 = lds_scale<ST>(s0p + nl * L::kSElt);
                const float sa1 = lds_scale<ST>(s0p + (nl + 8) * L::kSElt);
                if constexpr (kBias) {
#pragma unroll
                    for (int u = 0; u < kUPS; ++u) {
                        if (u >= nu) continue;
                        const float s0 = u ? lds_scale<ST>(s0p + L::kSUnit + nl * L::kSElt) : sa0;
                        const float s1 = u ? lds_scale<ST>(s0p + L::kSUnit + (nl + 8) * L::kSElt) : sa1;
                        const uint8_t* bp = stage + L::kB + u * L::kBUnit;
                        const float b0 = lds_scale<float>(bp + nl * 4), b1 = lds_scale<float>(bp + (nl + 8) * 4);
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            acc[j][m][0] += tacc[u][m][0] * s0 + xs[u][0][m][0] * b0;
                            acc[j][m][1] += tacc[u][m][1] * s0 + xs[u][0][m][1] * b0;
                            acc[j][m][2] += tacc[u][m][2] * s1 + xs[u][0][m][0] * b1;
                            acc[j][m][3] += tacc[u][m][3] * s1 + xs[u][0][m][1] * b1;
                        }
                    }
                } else if (same) {
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        acc[j][m][0] = fmaf(tacc[0][m][0] + tacc[1][m][0], sa0, acc[j][m][0]);
                        acc[j][m][1] = fmaf(tacc[0][m][1] + tacc[1][m][1], sa0, acc[j][m][1]);
                        acc[j][m][2] = fmaf(tacc[0][m][2] + tacc[1][m][2], sa1, acc[j][m][2]);
                        acc[j][m][3] = fmaf(tacc[0][m][3] + tacc[1][m][3], sa1, acc[j][m][3]);
                    }
                } else {
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        acc[j][m][0] = fmaf(tacc[0][m][0], sa0, acc[j][m][0]);
                        acc[j][m][1] = fmaf(tacc[0][m][1], sa0, acc[j][m][1]);
                        acc[j][m][2] = fmaf(tacc[0][m][2], sa1, acc[j][m][2]);
                        acc[j][m][3] = fmaf(tacc[0][m][3], sa1, acc[j][m][3]);
                    }
                    if (nu == 2) {
                        const float sb0 = lds_scale<ST>(s0p + L::kSUnit + nl * L::kSElt);
                        const float sb1 = lds_scale<ST>(s0p + L::kSUnit + (nl + 8) * L::kSElt);
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            acc[j][m][0] = fmaf(tacc[1][m][0], sb0, acc[j][m][0]);
                            acc[j][m][1] = fmaf(tacc[1][m][1], sb0, acc[j][m][1]);
                            acc[j][m][2] = fmaf(tacc[1][m][2], sb1, acc[j][m][2]);
                            acc[j][m][3] = fmaf(tacc[1][m][3], sb1, acc[j][m][3]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
    }

    // ------------------------------------------------------------- epilogue
    OT* C = reinterpret_cast<OT*>(p.C);
    // Store a float4 of the fragment (strip sl, token tile m, lane) to C.
    auto store_frag = [&](int sl, int m, int ln, float4 v) {
        if (sl >= width) return;
        const int n = sg * kGroupCols + sl * kStripCols + (ln >> 2);
        const int tok = 8 * m + 2 * (ln & 3);
        if (tok < p.M) {
            C[(size_t)tok * p.N + n] = from_f32<OT>(v.x);
            C[(size_t)tok * p.N + n + 8] = from_f32<OT>(v.z);
        }
        if (tok + 1 < p.M) {
            C[(size_t)(tok + 1) * p.N + n] = from_f32<OT>(v.y);
            C[(size_t)(tok + 1) * p.N + n + 8] = from_f32<OT>(v.w);
        }
    };
    if (cs == 1) {
        if (warp < kConsumerWarps) {
#pragma unroll
            for (int j = 0; j < kStripsPerWarp; ++j)
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    store_frag(kStripsPerWarp * warp + j, m, lane,
                               make_float4(acc[j][m][0], acc[j][m][1], acc[j][m][2], acc[j][m][3]));
        }
        return;
    }
    // Cluster split-K: partial fragments to this CTA's shared memory (the ring,
    // idle now: every issued copy has landed and been consumed), cluster
    // barrier, then CTA `rank` reduces its 1/cs share over all cs CTAs in rank
    // order and writes C; a second barrier keeps every CTA's shared memory
    // alive until all remote reads are done.
    constexpr int kFrags = kConsumerWarps * kStripsPerWarp * MT * 32;  // float4 per CTA
    const uint32_t red = smem_u32(ring);
    __syncthreads();
    if (warp < kConsumerWarps) {
#pragma unroll
        for (int j = 0; j < kStripsPerWarp; ++j)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int i = ((warp * kStripsPerWarp + j) * MT + m) * 32 + lane;
                sts_f4(red + 16 * i, make_float4(acc[j][m][0], acc[j][m][1], acc[j][m][2], acc[j][m][3]));
            }
    }
    cluster_sync();
    const int share = (kFrags + cs - 1) / cs;  // cs need not divide kFrags
    for (int i = rank * share + (int)threadIdx.x; i < min(kFrags, (rank + 1) * share); i += kThreads) {
        float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < cs; ++q) {
            const float4 v = ld_dsmem_f4(mapa_shared(red + 16 * i, (uint32_t)q));
            s4.x += v.x;
            s4.y += v.y;
            s4.z += v.z;
            s4.w += v.w;
        }
        const int ln = i & 31, rest = i >> 5;
        const int m = rest % MT, wj = rest / MT;
        store_frag(wj, m, ln, s4);  // wj = warp * 2 + j = strip index
    }
    cluster_sync();
}

using KernelFn = void (*)(DecodeParams);

struct KernelInfo {
    KernelFn fn = nullptr;
    int smem = 0;
    bool x_tma = false;
};

template <int WBITS, int MT, typename AT, typename ST, typename OT, bool kBias, bool kG32, int kNStages>
KernelInfo kernel_info() {
    using L = Stage<WBITS, AT, ST, kBias, kG32, kNStages>;
    return {decode_kernel<WBITS, MT, AT, ST, OT, kBias, kG32, kNStages>, L::kSmem, L::kXTma};
}

// Output dtype: the activation's own 16-bit type or f32 (f32 activations: f32 out).
template <int WBITS, int MT, typename AT, typename ST, bool kBias, bool kG32 = false, int kNStages = 4>
KernelInfo pick_out(DType c) {
    if (c == DType::F32) return kernel_info<WBITS, MT, AT, ST, float, kBias, kG32, kNStages>();
    if constexpr (std::is_same<AT, __half>::value) {
        if (c == DType::F16) return kernel_info<WBITS, MT, AT, ST, __half, kBias, kG32, kNStages>();
    }
    if constexpr (std::is_same<AT, __nv_bfloat16>::value) {
        if (c == DType::BF16) return kernel_info<WBITS, MT, AT, ST, __nv_bfloat16, kBias, kG32, kNStages>();
    }
    return {};
}

// Group 32 at M <= 8: three stages let four CTAs share an SM (the two extra scale and
// bias rows make four stages too large for that), which pays on layers of >= 56 strip
// groups (Q4_K at M = 1: gate_up 46.4 -> 34.5 us, QKV 15.8 -> 11.8) and loses on
// narrower ones, whose clusters of 8-12 CTAs per strip group need the deeper ring
// (O 9.9 -> 11.4 us).
template <int MT, typename AT, bool kBias>
KernelInfo pick_g32(const GemmArgs& a) {
    if constexpr (MT == 1) {
        if (TileGeom(a.K, a.N, 4).NSG >= 56) return pick_out<4, MT, AT, float, kBias, true, 3>(a.c_dtype);
    }
    return pick_out<4, MT, AT, float, kBias, true, 4>(a.c_dtype);
}

// fp32 activations (group >= 64) at M <= 8: their padded activation rows make a stage
// ~19 KB, so four stages hold two or three CTAs per SM.  Three stages (one CTA more)
// pay on layers of < 56 strip groups (the reference's fp32 form, O at M = 1: 16.3 ->
// 11.5 us; down at M = 8: 39.1 -> 27.0) and lose on wider ones (QKV 16.7 -> 19.4).
template <int MT, typename ST, bool kBias>
KernelInfo pick_f32(const GemmArgs& a) {
    if constexpr (MT == 1) {
        if (TileGeom(a.K, a.N, 4).NSG < 56) return pick_out<4, MT, float, ST, kBias, false, 3>(a.c_dtype);
    }
    return pick_out<4, MT, float, ST, kBias, false, 4>(a.c_dtype);
}

// Supported (activation, scale, bias) combinations.  int4: (f16,f16), (bf16,bf16),
// (f16|bf16, f32), (f32, f32) with or without bias for f16/f32 activations, and
// (f32, f16).  Ternary: (f16,f16), (bf16,bf16), (f32, f16).  Group 32 (int4, f32 scales):
// f16 / f32 activations with or without bias, bf16 without.
template <int WBITS, int MT>
KernelInfo pick(const GemmArgs& a) {
    const bool bias = a.bias != nullptr;
    if (a.group % kBlockK) {
        if constexpr (WBITS == 4) {
            if (a.group != 32 || a.s_dtype != DType::F32) return {};
            if (a.a_dtype == DType::F16) return bias ? pick_g32<MT, __half, true>(a) : pick_g32<MT, __half, false>(a);
            if (a.a_dtype == DType::BF16 && !bias) return pick_g32<MT, __nv_bfloat16, false>(a);
            if (a.a_dtype == DType::F32) return bias ? pick_g32<MT, float, true>(a) : pick_g32<MT, float, false>(a);
        }
        return {};
    }
    if (a.a_dtype == DType::F16 && a.s_dtype == DType::F16 && !bias)
        return pick_out<WBITS, MT, __half, __half, false>(a.c_dtype);
    if (a.a_dtype == DType::BF16 && a.s_dtype == DType::BF16 && !bias)
        return pick_out<WBITS, MT, __nv_bfloat16, __nv_bfloat16, false>(a.c_dtype);
    if constexpr (WBITS == 2) {
        // fp32 activations (two fp16 terms) on ternary weights with fp16 scales:
        // TQ1_0 layers converted at load (hq_tq1_0_to_tile_t2) with the reference's fp32 x
        if (a.a_dtype == DType::F32 && a.s_dtype == DType::F16 && !bias)
            return pick_out<WBITS, MT, float, __half, false>(a.c_dtype);
    }
    if constexpr (WBITS == 4) {
        if (a.a_dtype == DType::F16 && a.s_dtype == DType::F32)
            return bias ? pick_out<WBITS, MT, __half, float, true>(a.c_dtype)
                        : pick_out<WBITS, MT, __half, float, false>(a.c_dtype);
        if (a.a_dtype == DType::BF16 && a.s_dtype == DType::F32 && !bias)
            return pick_out<WBITS, MT, __nv_bfloat16, float, false>(a.c_dtype);
        if (a.a_dtype == DType::F32 && a.s_dtype == DType::F32)
            return bias ? pick_f32<MT, float, true>(a) : pick_f32<MT, float, false>(a);
        if (a.a_dtype == DType::F32 && a.s_dtype == DType::F16 && !bias) return pick_f32<MT, __half, false>(a);
    }
    return {};
}

KernelInfo select_kernel(const GemmArgs& a) {
    const int MT = a.M <= 8 ? 1 : 2;
    if (a.wbits == 4) return MT == 1 ? pick<4, 1>(a) : pick<4, 2>(a);
    return MT == 1 ? pick<2, 1>(a) : pick<2, 2>(a);
}

// CTAs per strip group, from {1, 2, 4, 8, 10, 12} (<= KB): the cs minimising
// resident waves x k-blocks per CTA plus a reduction cost that grows with cs,
// using the measured cluster occupancy of this kernel.  Narrow layers (N = 5120:
// 40 strip groups) need clusters of more than 8 CTAs to put enough bytes in
// flight per SM; larger clusters (14, 16) measured slower on B200.
int cluster_size(const void* fn, int smem, int N, int K, int wbits, int dev) {
    const TileGeom geo(K, N, wbits);
    static const int kCandidates[] = {1, 2, 4, 8, 10, 12};
    int best = 1;
    long long best_cost = -1;
    for (int cs : kCandidates) {
        if (cs > geo.KB) break;
        const int clusters = max_active_clusters(fn, kThreads, smem, cs, dev);
        if (clusters <= 0) continue;
        const long long waves = (geo.NSG + clusters - 1) / clusters;
        const long long cost = waves * ((geo.KB + cs - 1) / cs) * 8 + 8 * cs;
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = cs;
        }
    }
    return best;
}

bool g_early_weights = true;

// Smallest layer the integer-MMA stream kernel takes: in strip groups of 128
// columns for 16-bit activations, in (strip group, k-block) units for fp32; and
// its largest M (one tile of 4 token slots: at M = 8 the cluster kernel is
// faster, gate_up 27.8 us against 28.4).  The tcgen05 kernel's narrowest layer.
#ifndef HQ_DECODE_I8_MIN_NSG
#define HQ_DECODE_I8_MIN_NSG 128
#endif
#ifndef HQ_DECODE_I8_MIN_NSG_T2
#define HQ_DECODE_I8_MIN_NSG_T2 128
#endif
#ifndef HQ_DECODE_I8_MAX_M
#define HQ_DECODE_I8_MAX_M 4
#endif
#ifndef HQ_DECODE_TC_MIN_NSG
#define HQ_DECODE_TC_MIN_NSG 128
#endif
#ifndef HQ_DECODE_I8_MIN_UNITS_F32
#define HQ_DECODE_I8_MIN_UNITS_F32 8192
#endif

}  // namespace

void set_decode_launch_overlap(bool on) { g_early_weights = on; }

bool decode_supported(const GemmArgs& a) { return select_kernel(a).fn != nullptr; }

// Only the integer-MMA kernel (wide layers, int4 or ternary) keeps state in the workspace.
size_t decode_workspace_bytes(int M, int N, int K, int wbits, int dev) {
    (void)M;
    (void)wbits;
    return decode_i8_workspace_bytes(N, K, dev);
}

cudaError_t launch_decode(const GemmArgs& a) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (a.M < 1 || a.M > kMaxRows) return cudaErrorInvalidValue;
    // Wide layers (>= 128 strip groups) at M <= 4 with 16-bit activations stream
    // faster through the integer-MMA kernel (hq_decode_i8.cu; gate_up 5120 x
    // 34816: 26.2 us against 28.0 here): its consumer spends ~3x fewer
    // instructions per byte of codes.  Narrow layers, and M > 4, keep this
    // kernel, whose cluster split-K has a shorter start-up and tail.
    // fp32 activations take it for large layers (>= 8192 k-block units, 32 MB of
    // codes: 27B down 17408 x 5120 at 27.9 us against 42.0 here, gate_up 36.1
    // against 56.3): this kernel splits them into two fp16 halves and runs
    // twice the MMAs.  Smaller fp32 layers stay here (QKV 17.8 us against 19.4).
    const TileGeom tg(a.K, a.N, a.wbits);
    const bool g64 = a.group % kBlockK == 0;  // group 32 runs only here
    const bool i8_shape = g64 && (a.a_dtype == DType::F32 ? tg.units() >= HQ_DECODE_I8_MIN_UNITS_F32
                                  : a.wbits == 2          ? tg.NSG >= HQ_DECODE_I8_MIN_NSG_T2
                                                          : tg.NSG >= HQ_DECODE_I8_MIN_NSG);
    if (a.M <= HQ_DECODE_I8_MAX_M && i8_shape && decode_i8_supported(a)) return launch_decode_i8(a, g_early_weights);
    // M > 8 on wide layers (>= 128 strip groups) runs on tcgen05: the mma.sync
    // kernel needs two token tiles there and the tensor-memory kernel's cost does
    // not depend on M (gate_up at M = 16: 34.1 us against 47.1).  Narrower
    // layers stream faster here (QKV at M = 16: 15.2 us against 17.2).
    if (a.M > 8 && g64 && TileGeom(a.K, a.N, a.wbits).NSG >= HQ_DECODE_TC_MIN_NSG && decode_tc_supported(a))
        return launch_decode_tc(a, false);
    const TileGeom geo(a.K, a.N, a.wbits);
    const KernelInfo ki = select_kernel(a);
    if (!ki.fn) return cudaErrorInvalidValue;
    e = ensure_smem_attr(reinterpret_cast<const void*>(ki.fn), dev, ki.smem);
    if (e != cudaSuccess) return e;
    DecodeParams p;
    memset(&p, 0, sizeof p);
    if (ki.x_tma) {
        // [M][K] 16-bit activations; a box is 64 k x 16 rows, rows >= M read zero.
        e = make_tmap_2d(&p.x_map, a.A, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.M,
                         (uint64_t)a.K * 2, kBlockK, kMaxRows, CU_TENSOR_MAP_SWIZZLE_128B);
        if (e != cudaSuccess) return e;
    }
    p.A = a.A;
    p.W = a.W;
    p.S = a.S;
    p.bias = a.bias;
    p.C = a.C;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.group = a.group;
    p.err = device_error_word(dev);
    p.cs = cluster_size(reinterpret_cast<const void*>(ki.fn), ki.smem, a.N, a.K, a.wbits, dev);
    // Weights before griddepcontrol.wait only in the integer kernel: here the
    // early copies compete with the previous kernel's tail and measured slower
    // (27B down at M = 1: 18.6 us with them, 17.2 without; QKV 9.8 / 9.3; the
    // tcgen05 kernel: gate_up at M = 16 34.2 / 33.7).  The launch itself still
    // overlaps the previous kernel's tail (CTA start, barrier set-up).
    p.early_weights = 0;

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
