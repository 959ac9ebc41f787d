// hq_decode.cu -- HBM-streaming W4A16 / ternary GEMM for decode (M <= 16).
//
// Replaces kernel_marlin_gemm_int4_templated / _dynamic and the memset +
// atomicAdd split-K of the reference (hydrogen/src/model/marlin_gemm.cu:130-322,
// :556-601).  Design for B200:
//   * Byte-balanced persistent split ("stream-K").  The tile order stores the
//     weights as units (strip group sg, k-block kb) in sg-major order, each one
//     contiguous span, so the whole tensor is one byte stream.  The grid has
//     one CTA per SM and CTA c takes units [U c / G, U (c+1) / G): every SM
//     streams the same number of bytes whatever the shape, and a launch costs
//     one wave.  Shared memory (~105 KB) and registers are sized so that two
//     CTAs fit an SM: the next GEMM on the stream (programmatic dependent
//     launch) becomes resident beside this one and streams its first stages
//     while this one finishes, so back-to-back GEMMs keep HBM busy.
//   * One producer warp moves a stage -- up to 4 k-blocks (int4) / 8 (ternary)
//     of one strip group, 16 KB of codes -- with one 1-D bulk copy (TMA engine,
//     L2 evict-first), plus each k-block's activation tile (one 2-D TMA box of
//     64 k x 8 or 16 rows, 128-byte swizzled, rows >= M zero-filled) and its
//     scale (and bias) row, into a ring of several stages.  Weights and scales
//     are requested before griddepcontrol.wait, activations after it.
//   * Eight consumer warps; warp w owns strip w (16 output columns) of the
//     stage's strip group, so its partial sums never leave registers until the
//     group is done.  A lane's 16 bytes of a k-block are its A fragments for
//     four m16n8k16 steps: codes are OR-ed into an fp16/bf16 exponent pattern
//     and one packed subtract gives exact q; fp32 accumulation, the group
//     scale applied in fp32 per k-block.
//   * A strip group wholly inside one CTA's range is stored straight from
//     registers.  A group split between CTAs (at most the first and last of a
//     CTA's range) is finished by the last CTA to reach it: every sharer
//     writes its fp32 partial tile to the workspace and bumps the group's
//     counter; the CTA that brings the counter to the number of sharers sums
//     the partials in CTA order (deterministic: the same order whichever CTA
//     arrives last), writes C and resets the counter.  No CTA ever waits on
//     another, no memset, no float atomics.
#include "hq_common.cuh"
#include "hq_decode_frag.cuh"
#include "hq_internal.h"
#include "hq_layout.h"
#include "hq_tmap.h"

#include <algorithm>
#include <cstring>
#include <type_traits>

#ifndef HQ_DECODE_CTAS_PER_SM
#define HQ_DECODE_CTAS_PER_SM 1
#endif
#ifndef HQ_DECODE_RING_KB
#define HQ_DECODE_RING_KB 200
#endif
#ifndef HQ_DECODE_TC_ROUTE
#define HQ_DECODE_TC_ROUTE 1
#endif
#ifndef HQ_DECODE_I8
#define HQ_DECODE_I8 1
#endif

namespace hq {

namespace {

using frag::ComputeType;
using frag::lds_scale;
using frag::WFrag;
using frag::XFrag;
using frag::XFragF32;

constexpr int kNC = 16;  // consumer warps: warps w and w + 8 own strip w of a strip group
constexpr int kProducerWarps = 2;  // warp kNC issues the code copy; both share the small operands
constexpr int kProducerWarp = kNC;
constexpr int kThreads = (kNC + kProducerWarps) * 32;
constexpr int kMaxRows = 16;
constexpr int kCtasPerSm = HQ_DECODE_CTAS_PER_SM;
constexpr int kRingBudget = HQ_DECODE_RING_KB * 1024;
constexpr int kPairBar = 1;  // named barrier of all consumer warps
constexpr int kHalfBar = 2;  // named barrier of the first eight consumer warps
constexpr int kBatch = 4;     // k-blocks a consumer warp keeps in flight

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }
constexpr int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Shared-memory layout of one ring stage.
template <int WBITS, int MT, typename AT, typename ST, bool kBias>
struct Ring {
    static constexpr int kCB = WBITS == 4 ? 512 : 256;
    static constexpr int kUPS = WBITS == 4 ? 8 : 16;          // k-blocks per stage
    static constexpr int kW = kUPS * kGroupStrips * kCB;     // codes of a full-width stage: 32 KB, one bulk copy
    static constexpr bool kXTma = sizeof(AT) == 2;           // 16-bit activations: 128-byte XOR-swizzled rows
    static constexpr int kXRows = 8 * MT;
    static constexpr int kXRowBytes = kBlockK * (int)sizeof(AT);
    static constexpr int kXRow = kXTma ? 128 : XFragF32::kRowBytes;
    static constexpr int kXUnit = kXRows * kXRow;
    static constexpr int kSUnit = kGroupCols * (int)sizeof(ST);
    static constexpr int kBUnit = kBias ? kGroupCols * 4 : 0;
    static constexpr int kX = kW;
    static constexpr int kS = kX + kUPS * kXUnit;
    static constexpr int kB = kS + kUPS * kSUnit;
    static constexpr int kBytes = align_up(kB + kUPS * kBUnit, 128);
    static constexpr int kStages = clampi(kRingBudget / kBytes, 2, 8);
    static constexpr int kPair = 2 * 8 * MT * 32 * 16;  // two buffers of half 1's sums (float4 per lane)
    static constexpr int kSmem = kStages * kBytes + kPair + 128 /* base alignment slack */ + 2 * kStages * 8 + 16;
};

struct alignas(16) DecodeParams {
    const void* A;
    const uint8_t* W;
    const void* S;
    const float* bias;
    void* C;
    unsigned* err;       // device error word
    unsigned* counters;  // [NSG] arrivals per strip group (workspace; zero between calls)
    float4* partials;    // [G][2][kNC][MT * 32] fp32 partial fragments (workspace)
    int M, N, K, group;
    int early_weights;  // stream weights/scales before the previous kernel finishes
};

// One stage: k-blocks [kb, kb + n) of strip group sg.
struct Span {
    int sg, kb, n;
};

// The stage sequence of a unit range, identical for the producer and the
// consumers (incremental: no 64-bit division per stage).
struct Walker {
    int sg, kb, left, KB, ups;
    __device__ __forceinline__ Walker(long long u, long long end, int KB_, int ups_)
        : sg((int)(u / KB_)), kb((int)(u % KB_)), left((int)(end - u)), KB(KB_), ups(ups_) {}
    __device__ __forceinline__ bool next(Span& s) {
        if (left <= 0) return false;
        int n = KB - kb < ups ? KB - kb : ups;
        if (n > left) n = left;
        s.sg = sg;
        s.kb = kb;
        s.n = n;
        left -= n;
        kb += n;
        if (kb == KB) {
            kb = 0;
            ++sg;
        }
        return true;
    }
};

__device__ __forceinline__ long long range_begin(long long U, int G, int c) { return U * c / G; }

// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of(long long u, long long U, int G) {
    int c = (int)((u * G) / U);
    while (c + 1 < G && range_begin(U, G, c + 1) <= u) ++c;
    while (c > 0 && range_begin(U, G, c) > u) --c;
    return c;
}

template <int WBITS, int MT, typename AT, typename ST, typename OT, bool kBias>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    using L = Ring<WBITS, MT, AT, ST, kBias>;
    constexpr bool kSplit = std::is_same<AT, float>::value;
    constexpr bool kBF16 = ComputeType<AT>::bf16;  // float activations compute in fp16
    constexpr int kCB = L::kCB;
    constexpr int kLaneBytes = kCB / 32;
    constexpr int kStages = L::kStages;
    constexpr int kUPS = L::kUPS;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    float4* pair_buf = reinterpret_cast<float4*>(ring + kStages * L::kBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * L::kBytes + L::kPair);
    uint64_t* empty = full + kStages;
    volatile int* s_last = reinterpret_cast<volatile int*>(empty + kStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WBITS);
    const int KB = geo.KB;
    const long long U = geo.units();
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    const long long u_begin = range_begin(U, G, c), u_end = range_begin(U, G, c + 1);
    const int upg = p.group / kBlockK;  // k-blocks per scale group

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1 + 32 * kProducerWarps);  // the code copy's expect-tx + one cp.async arrival per producer lane
            mbar_init(&empty[i], kNC);
        }
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        pdl_launch_dependents();
    }
    __syncthreads();

    if (warp >= kProducerWarp) {
        // --------------------------------------------------------- producers
        // Warp kProducerWarp issues the stage's codes as one bulk copy; the small
        // operands (activation rows, scale and bias rows) go as 16-byte cp.async
        // spread over both producer warps, each lane then arriving once they land.
        const int pl = (warp - kProducerWarp) * 32 + lane;
        constexpr int kPL = 32 * kProducerWarps;
        const uint64_t pol = l2_policy_evict_first();
        const uint8_t* Ab = reinterpret_cast<const uint8_t*>(p.A);
        const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
        const uint8_t* Bb = reinterpret_cast<const uint8_t*>(p.bias);
        const int xrows = p.M < L::kXRows ? p.M : L::kXRows;  // rows >= M feed only unstored MMA columns
        auto stage_ptr = [&](int it) { return ring + (it % kStages) * L::kBytes; };
        // Codes, scales and biases of stage `it` (no earlier kernel writes them).
        auto issue_w = [&](int it, const Span& d) {
            const int slot = it % kStages;
            uint8_t* st = stage_ptr(it);
            const int width = geo.width(d.sg);
            const int s_chunks = width * kStripCols * (int)sizeof(ST) / 16;
            const int b_chunks = kBias ? width * kStripCols * 4 / 16 : 0;
            const uint32_t wbytes = (uint32_t)d.n * (uint32_t)width * kCB;
            if (pl == 0) {
                mbar_arrive_expect_tx(&full[slot], wbytes);
                bulk_g2s_hint(st, p.W + geo.unit_offset((long long)d.sg * KB + d.kb), wbytes, &full[slot], pol);
            }
            // one scale (and bias) row per k-block: [group][the group's columns]
            for (int i = pl; i < d.n * (s_chunks + b_chunks); i += kPL) {
                const int r = i / (s_chunks + b_chunks), cc = i - r * (s_chunks + b_chunks);
                const size_t off = (size_t)((d.kb + r) / upg) * p.N + (size_t)d.sg * kGroupCols;
                if (cc < s_chunks)
                    cp_async16(st + L::kS + r * L::kSUnit + 16 * cc, Sb + off * sizeof(ST) + 16 * cc);
                else if constexpr (kBias)
                    cp_async16(st + L::kB + r * L::kBUnit + 16 * (cc - s_chunks), Bb + off * 4 + 16 * (cc - s_chunks));
            }
        };
        // Activation rows of stage `it` (may depend on the previous kernel), then
        // this lane's arrival once its copies of the stage have landed.
        auto issue_x = [&](int it, const Span& d) {
            const int slot = it % kStages;
            uint8_t* st = stage_ptr(it);
            constexpr int kRowChunks = kBlockK * (int)sizeof(AT) / 16;  // 16-byte pieces of one row of one k-block
            const int per_kb = xrows * kRowChunks;
            for (int i = pl; i < d.n * per_kb; i += kPL) {
                const int u = i / per_kb, rem = i - u * per_kb, r = rem / kRowChunks, cc = rem - r * kRowChunks;
                const uint8_t* src = Ab + ((size_t)r * p.K + (size_t)(d.kb + u) * kBlockK) * sizeof(AT) + 16 * cc;
                uint8_t* dst = st + L::kX + u * L::kXUnit;
                if constexpr (L::kXTma)
                    dst += r * 128 + ((cc ^ (r & 7)) << 4);  // 128-byte rows, XOR-swizzled 16-byte chunks
                else
                    dst += r * L::kXRow + 16 * cc;
                cp_async16(dst, src);
            }
            cp_async_mbar_arrive(&full[slot]);
        };
        Walker wk(u_begin, u_end, KB, kUPS);
        Span d;
        Span pend[kStages];
        int it = 0;
        // First pass over the ring: every slot is free.  Codes first; activations
        // once the previous kernel has finished.
        if (!p.early_weights) pdl_wait();
        while (it < kStages && wk.next(d)) {
            issue_w(it, d);
            if (p.early_weights)
                pend[it] = d;
            else
                issue_x(it, d);
            ++it;
        }
        if (p.early_weights) {
            pdl_wait();
            for (int j = 0; j < it; ++j) issue_x(j, pend[j]);
        }
        while (wk.next(d)) {
            const int slot = it % kStages;
            int w_ok = 1;
            if (lane == 0) w_ok = mbar_wait(&empty[slot], ((uint32_t)(it / kStages) & 1u) ^ 1u, p.err);
            w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
            if (!w_ok) break;
            issue_w(it, d);
            issue_x(it, d);
            ++it;
        }
        // Copies still in flight land before the CTA exits.
        if (lane == 0)
            for (int j = it - kStages < 0 ? 0 : it - kStages; j < it; ++j)
                mbar_wait(&full[j % kStages], (uint32_t)(j / kStages) & 1u, p.err);
        __syncwarp();
        return;
    }

    // ------------------------------------------------------------ consumers
    // Two warps per strip: half 0 takes the first half of every stage's
    // k-blocks, half 1 the second; their sums meet in shared memory when a
    // strip group is done.
    pdl_wait();
    const int g = lane >> 2, t = lane & 3;
    const int sl = warp & 7, half = warp >> 3;
    using XF = typename std::conditional<kSplit, XFragF32, XFrag<AT>>::type;
    const uint32_t kOnes = 0x3C003C00u;  // fp16 (1, 1) for the bias row sums
    OT* C = reinterpret_cast<OT*>(p.C);

    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][i] = 0.f;

    auto store_frag = [&](int sg, int m, float4 v) {
        const int n = sg * kGroupCols + sl * kStripCols + g;
        const int tok = 8 * m + 2 * t;
        if (tok < p.M) {
            C[(size_t)tok * p.N + n] = from_f32<OT>(v.x);
            C[(size_t)tok * p.N + n + 8] = from_f32<OT>(v.z);
        }
        if (tok + 1 < p.M) {
            C[(size_t)(tok + 1) * p.N + n] = from_f32<OT>(v.y);
            C[(size_t)(tok + 1) * p.N + n + 8] = from_f32<OT>(v.w);
        }
    };

    // A batch of up to kBatch k-blocks (from k-block u0 of the stage) of this
    // warp's strip: all code and scale loads first, then independent MMA chains
    // per k-block (so the loads, the dequant and the tensor-core latencies of
    // different k-blocks overlap), then the scales.  kFull (a whole batch, the
    // common case) is straight-line code; otherwise k-blocks u >= n are skipped
    // by warp-uniform branches.
    auto consume_batch = [&](const uint8_t* stage, int u0, int width, int n, auto full_tag) {
        constexpr bool kFull = decltype(full_tag)::value;
        constexpr int kUPS = kBatch;
        const uint32_t unit_bytes = (uint32_t)width * kCB;
        const int nl = sl * kStripCols + g;  // column within the group
        uint4 wv[kUPS];
        float sc0[kUPS], sc1[kUPS];
#pragma unroll
        for (int u = 0; u < kUPS; ++u) {
            const bool on = kFull || u < n;
            const uint8_t* wp = stage + (u0 + u) * unit_bytes + sl * kCB + lane * kLaneBytes;
            if constexpr (WBITS == 4) {
                wv[u] = on ? *reinterpret_cast<const uint4*>(wp) : make_uint4(0u, 0u, 0u, 0u);
            } else {
                const uint2 v = on ? *reinterpret_cast<const uint2*>(wp) : make_uint2(0u, 0u);
                wv[u] = make_uint4(v.x, v.y, 0u, 0u);
            }
            const uint8_t* sp = stage + L::kS + (u0 + u) * L::kSUnit;
            sc0[u] = on ? lds_scale<ST>(sp + nl * sizeof(ST)) : 0.f;
            sc1[u] = on ? lds_scale<ST>(sp + (nl + 8) * sizeof(ST)) : 0.f;
        }
        float tacc[kUPS][MT][4];
        float xs[kUPS][MT][4];
#pragma unroll
        for (int u = 0; u < kUPS; ++u) {
#pragma unroll
            for (int m = 0; m < MT; ++m)
#pragma unroll
                for (int i = 0; i < 4; ++i) tacc[u][m][i] = xs[u][m][i] = 0.f;
            if (!kFull && u >= n) continue;
            const uint8_t* tile = stage + L::kX + (u0 + u) * L::kXUnit;
            WFrag<WBITS, kBF16, kBias> wf;
            wf.build(wv[u]);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                XF xf;
                xf.load(tile, 8 * m + g, t);
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    if constexpr (kSplit) {
                        mma_16816<false>(tacc[u][m], wf.r[s], xf.hi[2 * s], xf.hi[2 * s + 1]);
                        mma_16816<false>(tacc[u][m], wf.r[s], xf.lo[2 * s], xf.lo[2 * s + 1]);
                    } else {
                        mma_16816<kBF16>(tacc[u][m], wf.r[s], xf.b0(s), xf.b1(s));
                    }
                }
                if constexpr (kBias) {
                    // Row sums of the activations (a ones A operand): the bias term b * sum(x).
                    const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        if constexpr (kSplit) {
                            mma_16816<false>(xs[u][m], ones, xf.hi[2 * s], xf.hi[2 * s + 1]);
                            mma_16816<false>(xs[u][m], ones, xf.lo[2 * s], xf.lo[2 * s + 1]);
                        } else {
                            mma_16816<kBF16>(xs[u][m], ones, xf.b0(s), xf.b1(s));
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kUPS; ++u) {
            if (!kFull && u >= n) continue;
            float b0 = 0.f, b1 = 0.f;
            if constexpr (kBias) {
                const uint8_t* bp = stage + L::kB + (u0 + u) * L::kBUnit;
                b0 = lds_scale<float>(bp + nl * 4);
                b1 = lds_scale<float>(bp + (nl + 8) * 4);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                acc[m][0] = fmaf(tacc[u][m][0], sc0[u], acc[m][0]);
                acc[m][1] = fmaf(tacc[u][m][1], sc0[u], acc[m][1]);
                acc[m][2] = fmaf(tacc[u][m][2], sc1[u], acc[m][2]);
                acc[m][3] = fmaf(tacc[u][m][3], sc1[u], acc[m][3]);
                if constexpr (kBias) {
                    acc[m][0] = fmaf(xs[u][m][0], b0, acc[m][0]);
                    acc[m][1] = fmaf(xs[u][m][1], b0, acc[m][1]);
                    acc[m][2] = fmaf(xs[u][m][2], b1, acc[m][2]);
                    acc[m][3] = fmaf(xs[u][m][3], b1, acc[m][3]);
                }
            }
        }
    };

    const int first_sg = (int)(u_begin / KB);
    int pend_sg[2] = {-1, -1};  // strip groups handed to the fixup, by slot
    int nflush = 0;
    // Strip group `sg` is done for this CTA: half 1 hands its sums to half 0,
    // which stores the group or, when other CTAs share it, writes the partial
    // and lets thread 0 count the arrival (the last arriver sums after the loop).
    auto flush_group = [&](int sg) {
        float4* xch = pair_buf + ((nflush & 1) * 8 + sl) * (MT * 32);
        ++nflush;
        if (half == 1) {
#pragma unroll
            for (int m = 0; m < MT; ++m) xch[m * 32 + lane] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
        }
        named_bar_sync(kPairBar, kNC * 32);
        if (half == 0) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float4 v = xch[m * 32 + lane];
                acc[m][0] += v.x;
                acc[m][1] += v.y;
                acc[m][2] += v.z;
                acc[m][3] += v.w;
            }
            const int width = geo.width(sg);
            const long long g0 = (long long)sg * KB, g1 = g0 + KB;
            if (g0 >= u_begin && g1 <= u_end) {
                if (sl < width)
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        store_frag(sg, m, make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]));
            } else {
                const int slot = sg == first_sg ? 0 : 1;
                float4* mine = p.partials + (((size_t)c * 2 + slot) * 8 + sl) * (MT * 32);
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    mine[m * 32 + lane] = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
                named_bar_sync(kHalfBar, 8 * 32);
                if (threadIdx.x == 0) {
                    __threadfence();  // cumulative: orders every half-0 partial before the arrival
                    const int c_first = cta_of(g0, U, G), c_last = cta_of(g1 - 1, U, G);
                    const unsigned old = atomicAdd(&p.counters[sg], 1u);
                    s_last[slot] = old == (unsigned)(c_last - c_first);
                }
                pend_sg[slot] = sg;
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[m][i] = 0.f;
    };

    // After a timed-out wait the warp stops waiting but keeps the same control
    // flow (results are garbage, the error word is set): every thread still
    // reaches the barriers, so nothing hangs.
    bool waits_ok = true;
    Walker wk(u_begin, u_end, KB, kUPS);
    Span d;
    int it = 0, cur = -1;
    constexpr int kHalfUnits = kUPS / 2;
    while (wk.next(d)) {
        if (d.sg != cur) {
            if (cur >= 0) flush_group(cur);
            cur = d.sg;
        }
        const int slot = it % kStages;
        if (waits_ok) waits_ok = mbar_wait(&full[slot], (uint32_t)(it / kStages) & 1u, p.err);
        const uint8_t* stage = ring + slot * L::kBytes;
        const int width = geo.width(d.sg);
        if (sl < width) {
#pragma unroll
            for (int b = 0; b < kHalfUnits; b += kBatch) {
                const int u0 = half * kHalfUnits + b;
                const int nb = d.n - u0;
                if (nb >= kBatch)
                    consume_batch(stage, u0, width, kBatch, std::true_type{});
                else if (nb > 0)
                    consume_batch(stage, u0, width, nb, std::false_type{});
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++it;
    }
    if (cur >= 0) flush_group(cur);

    // Strip groups shared with other CTAs that this CTA reached last: sum every
    // sharer's partial in CTA order, store, and reset the group's counter.
    if (half == 0) {
        named_bar_sync(kHalfBar, 8 * 32);  // thread 0's arrival results are visible
#pragma unroll
        for (int slot = 0; slot < 2; ++slot) {
            const int sg = pend_sg[slot];
            if (sg < 0 || !s_last[slot]) continue;
            __threadfence();
            const long long g0 = (long long)sg * KB, g1 = g0 + KB;
            const int c_first = cta_of(g0, U, G), c_last = cta_of(g1 - 1, U, G);
            float4 sum[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) sum[m] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = c_first; q <= c_last; ++q) {
                const int qslot = (int)(range_begin(U, G, q) / KB) == sg ? 0 : 1;
                const float4* src = p.partials + (((size_t)q * 2 + qslot) * 8 + sl) * (MT * 32);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const float4 v = __ldcg(src + m * 32 + lane);
                    sum[m].x += v.x;
                    sum[m].y += v.y;
                    sum[m].z += v.z;
                    sum[m].w += v.w;
                }
            }
            if (sl < geo.width(sg))
#pragma unroll
                for (int m = 0; m < MT; ++m) store_frag(sg, m, sum[m]);
            if (threadIdx.x == 0) p.counters[sg] = 0u;
        }
    }
}

using KernelFn = void (*)(DecodeParams);

struct KernelInfo {
    KernelFn fn = nullptr;
    int smem = 0;
    bool x_tma = false;
    int x_rows = 0;
};

template <int WBITS, int MT, typename AT, typename ST, typename OT, bool kBias>
KernelInfo kernel_info() {
    using L = Ring<WBITS, MT, AT, ST, kBias>;
    return {decode_kernel<WBITS, MT, AT, ST, OT, kBias>, L::kSmem, L::kXTma, L::kXRows};
}

// Output dtype: the activation's own 16-bit type or f32 (f32 activations: f32 out).
template <int WBITS, int MT, typename AT, typename ST, bool kBias>
KernelInfo pick_out(DType c) {
    if (c == DType::F32) return kernel_info<WBITS, MT, AT, ST, float, kBias>();
    if constexpr (std::is_same<AT, __half>::value) {
        if (c == DType::F16) return kernel_info<WBITS, MT, AT, ST, __half, kBias>();
    }
    if constexpr (std::is_same<AT, __nv_bfloat16>::value) {
        if (c == DType::BF16) return kernel_info<WBITS, MT, AT, ST, __nv_bfloat16, kBias>();
    }
    return {};
}

// Supported (activation, scale, bias) combinations.  int4: (f16,f16), (bf16,bf16),
// (f16|bf16, f32), (f32, f32) with or without bias for f16/f32 activations, and
// (f32, f16).  Ternary: (f16,f16), (bf16,bf16).
template <int WBITS, int MT>
KernelInfo pick(const GemmArgs& a) {
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
    return {};
}

KernelInfo select_kernel(const GemmArgs& a) {
    const int MT = a.M <= 8 ? 1 : 2;
    if (a.wbits == 4) return MT == 1 ? pick<4, 1>(a) : pick<4, 2>(a);
    return MT == 1 ? pick<2, 1>(a) : pick<2, 2>(a);
}

int grid_ctas(int N, int K, int wbits, int dev) {
    const long long U = TileGeom(K, N, wbits).units();
    const long long G = (long long)device_info(dev).sm_count * kCtasPerSm;
    return (int)(U < G ? U : G);
}

size_t counters_bytes(int N) {
    const size_t nsg = (size_t)((N / kStripCols + kGroupStrips - 1) / kGroupStrips);
    return (nsg * 4 + 255) & ~(size_t)255;
}

bool g_early_weights = true;

}  // namespace

void set_decode_launch_overlap(bool on) { g_early_weights = on; }

bool decode_supported(const GemmArgs& a) { return select_kernel(a).fn != nullptr; }

// Arrival counters (one per strip group) followed by the partial tiles of the
// split strip groups: two per CTA, eight warps x 2 token tiles x 32 lanes x 16 B.
size_t decode_counters_bytes(int N) { return counters_bytes(N); }

size_t decode_split_bytes(int N, int K, int wbits, int dev) {
    const size_t G = (size_t)grid_ctas(N, K, wbits, dev);
    return counters_bytes(N) + G * 2 * kNC * 2 * 32 * sizeof(float4);
}

size_t decode_workspace_bytes(int M, int N, int K, int wbits, int dev) {
    (void)M;
    return decode_split_bytes(N, K, wbits, dev) + (wbits == 4 ? decode_i8_extra_bytes(K) : 0);
}

cudaError_t launch_decode(const GemmArgs& a) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (a.M < 1 || a.M > kMaxRows) return cudaErrorInvalidValue;
#if HQ_DECODE_I8
    // int4 codes x 16-bit activations, no bias: the integer tensor-core kernel.
    if (decode_i8_supported(a)) return launch_decode_i8(a, g_early_weights);
#endif
#if HQ_DECODE_TC_ROUTE
    // M > 8 on wide layers may run on tcgen05 (its cost does not depend on M).
    if (a.M > 8 && TileGeom(a.K, a.N, a.wbits).NSG >= 48 && decode_tc_supported(a))
        return launch_decode_tc(a, g_early_weights);
#endif
    const KernelInfo ki = select_kernel(a);
    if (!ki.fn) return cudaErrorInvalidValue;
    if (!a.ws || a.ws_bytes < decode_workspace_bytes(a.M, a.N, a.K, a.wbits, dev)) return cudaErrorInvalidValue;
    e = ensure_smem_attr(reinterpret_cast<const void*>(ki.fn), dev, ki.smem);
    if (e != cudaSuccess) return e;
    DecodeParams p;
    memset(&p, 0, sizeof p);
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
    p.counters = reinterpret_cast<unsigned*>(a.ws);
    p.partials = reinterpret_cast<float4*>(a.ws + counters_bytes(a.N));
    p.early_weights = (g_early_weights && !a.weights_just_written) ? 1 : 0;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid_ctas(a.N, a.K, a.wbits, dev));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)ki.smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, ki.fn, p);
}

}  // namespace hq
