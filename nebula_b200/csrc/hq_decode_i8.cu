// hq_decode_i8.cu -- decode GEMM (M <= 8) on the integer tensor cores:
// int4 (or ternary) codes x fixed-point activations through mma.sync
// s8 x s8 -> s32 (u8 x s8 for ternary).
//
// Replaces the reference's kernel_marlin_gemm_int4_templated / _dynamic and
// its memset + atomicAdd split-K (hydrogen/src/model/marlin_gemm.cu:130-322,
// :556-601) for the calls the dispatcher (hq_decode.cu) sends here: fp16 /
// bf16 activations, fp32 activations (two fixed-point parts), fp32 scales with
// the reference's bias, and this library's 2-bit ternary tiles.
//
// Why integers: a decode GEMM reads every weight byte once, so its speed is set
// by how few instructions turn a byte of codes into tensor-core operands.
// Expanding int4 into fp16 pairs costs ~9 instructions per 32-bit word.  Here:
//   * A weight byte pair of nibbles becomes two signed bytes 16 q (q = u - 8):
//     hi = (w & 0xF0F0F0F0) ^ 0x80808080 is the high nibble of every byte as
//     16 u - 128 = 16 q (one LOP3); the low nibbles take a shift first.  Both
//     classes carry the same factor 16, so they share one accumulator, and no
//     offset correction is needed (the MMA sees q itself).
//   * Activations are converted once per call by x_prep_kernel into two
//     signed-byte pieces of a 15-bit fixed-point copy: x = 2^-s (256 h + l)
//     with s per (token, scale group) chosen from the group's max|x|, h in
//     [-64, 64], l in [-128, 127].  Piece h of token m is MMA column 2m, piece
//     l column 2m + 1, so a lane holds both pieces of one token and combines
//     them exactly in int32 (256 c0 + c1).  The pieces are stored per k-block
//     in the order in which each lane's B fragments read them (one 16-byte
//     shared-memory load per lane per k-block and 4-token tile).
//   * The exact int32 sums are scaled once per scale group:
//     y += scale[g][n] * 2^-s / 16 * (256 c0 + c1), fp32.
// The fixed-point copy keeps 15 bits relative to the largest |x| of each
// (token, scale group): results stay within ~1e-5 of max|y| of the fp32
// dequantize-then-matmul.  A group holding Inf/NaN activations makes that
// token's outputs NaN.
//
// Streaming.  The tile order stores the weights as units (strip group sg,
// k-block kb) in sg-major order, each one contiguous span, so the tensor is one
// byte stream; CTA c of G (two per SM) takes units [U c / G, U (c+1) / G), an
// equal byte share whatever the shape.  A stage is up to 8 k-blocks of one
// strip group: its 32 KB of codes arrive as ONE bulk copy (the TMA engine
// charges a fixed cost per operation: 4 KB copies stream at a quarter of the
// rate of 32 KB ones), while the small operands -- activation pieces, weight-
// and activation-scale rows -- go as 16-byte cp.async spread over two producer
// warps (a warp holding many DRAM-latency cp.async per lane stalls its issue).
// Codes and weight scales are requested before griddepcontrol.wait,
// activation pieces after it.  Eight consumer warps each own one 16-column
// strip.  A strip group shared between CTAs is finished by the last CTA to
// arrive: every sharer writes its fp32 partial, one thread fences and counts
// the arrival, and the CTA that completes the count sums the partials in CTA
// order after its main loop (deterministic) and resets the counter.  No CTA
// waits on another; the workspace is zero-filled once, never per call.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"

#include <cstring>
#include <type_traits>
#include <utility>

// Two CTAs per SM, each with a ~100 KB ring of two 32 KB-code stages, eight
// consumer warps (one per strip) and two producer warps: measured fastest on
// B200 among 1-2 CTAs per SM x 8-16 consumer warps x 1-4 producer warps.
#ifndef HQ_DECODE_I8_CTAS_PER_SM
#define HQ_DECODE_I8_CTAS_PER_SM 2
#endif
#ifndef HQ_DECODE_I8_RING_KB
#define HQ_DECODE_I8_RING_KB 100
#endif
#ifndef HQ_DECODE_I8_CONSUMERS
#define HQ_DECODE_I8_CONSUMERS 8
#endif
#ifndef HQ_DECODE_I8_PRODUCERS
#define HQ_DECODE_I8_PRODUCERS 2
#endif
#ifndef HQ_DECODE_I8_UPS
#define HQ_DECODE_I8_UPS 8
#endif


namespace hq {

namespace {

constexpr int kNC = HQ_DECODE_I8_CONSUMERS;  // consumer warps: warps w, w + 8, ... own strip w of a strip group
constexpr int kHalves = kNC / 8;             // warps per strip, each taking 1/kHalves of every stage
constexpr int kProducerWarps = HQ_DECODE_I8_PRODUCERS;  // warp kNC issues the code copy; all share the small operands
static_assert(kNC == 8 || kNC == 16, "one or two consumer warps per strip");
constexpr int kProducerWarp = kNC;
constexpr int kThreads = (kNC + kProducerWarps) * 32;
constexpr int kUPS = HQ_DECODE_I8_UPS;  // k-blocks per stage (4 KB of full-group codes each: one bulk copy)
constexpr int kBatch = 4;      // k-blocks a consumer warp keeps in flight
constexpr int kTokTile = 4;    // tokens per MMA n-tile (two pieces each)
constexpr int kTileBytes = 512;  // piece bytes of one k-block and one 4-token tile
constexpr int kCtasPerSm = HQ_DECODE_I8_CTAS_PER_SM;
constexpr int kRingBudget = HQ_DECODE_I8_RING_KB * 1024;
constexpr int kPairBar = 1;  // named barrier of all consumer warps
constexpr int kHalfBar = 2;  // named barrier of the first eight consumer warps
constexpr int kPrepThreads = 256;  // 16 token slots x 16 threads

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }
constexpr int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Stage layout.  With fp32 scales the stage also carries, per scale group, the
// activation sums of the 16 token slots and the group's fp32 bias row (the
// reference's u * s + b form; read only when the call has a bias).
template <int NT, int WB, typename ST>
struct RingI8 {
    static constexpr bool kBias = std::is_same<ST, float>::value;
    static constexpr int kW = kUPS * kGroupStrips * (WB == 4 ? 512 : 256);  // codes
    static constexpr int kXUnit = NT * kTileBytes;       // pieces of one k-block
    static constexpr int kX = kW;
    static constexpr int kSUnit = kGroupCols * (int)sizeof(ST);  // one scale row of the group's columns
    static constexpr int kS = kX + kUPS * kXUnit;
    static constexpr int kXS = kS + kUPS * kSUnit;  // x scales: 16 token slots x fp32 per scale group
    static constexpr int kXQ = kXS + kUPS * 64;     // x sums: 16 token slots x fp32 per scale group
    static constexpr int kB = kXQ + (kBias ? kUPS * 64 : 0);  // bias rows (fp32), as the scale rows
    static constexpr int kXK = kB + (kBias ? kUPS * kSUnit : 0);  // ternary: x sums per (k-block, token slot), int
    static constexpr int kBytes = align_up(kXK + (WB == 2 ? kUPS * 64 : 0), 128);
    static constexpr int kStages = clampi(kRingBudget / kBytes, 2, 8);
    static constexpr int kPair = kHalves > 1 ? 2 * 8 * NT * 32 * 8 : 0;  // two buffers of half 1's sums (float2 per lane)
    static constexpr int kSmem = kStages * kBytes + kPair + 128 + 2 * kStages * 8 + 16;
};

struct alignas(16) I8Params {
    const uint8_t* W;
    const void* S;
    const float* bias;     // [K/group][N] fp32, or null
    const int8_t* pieces;  // [K/64][NT*4 tokens][2][4][16] (workspace)
    const float* xscale;   // [K/group][16] 2^-s per (group, token slot) (workspace)
    const float* xsum;     // [K/group][16] sum of x per (group, token slot) (workspace; read with a bias)
    const int* xkb;        // ternary: [K/64][16] sum of the fixed-point x per (k-block, token slot) (workspace)
    void* C;
    unsigned* err;
    unsigned* counters;  // [NSG]
    float2* partials;    // [G][2][8 strips][NT * 32]
    int M, N, K, group;
    int early_weights;
};

struct Span {
    int sg, kb, n;
};

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

__device__ __forceinline__ int cta_of(long long u, long long U, int G) {
    int c = (int)((u * G) / U);
    while (c + 1 < G && range_begin(U, G, c + 1) <= u) ++c;
    while (c > 0 && range_begin(U, G, c) > u) --c;
    return c;
}

// D (16x8 s32) += A (16x32 s8) x B (32x8 s8).
__device__ __forceinline__ void imma_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16 q as signed bytes from the high / low nibble of every byte of a tile word.
__device__ __forceinline__ uint32_t q16_hi(uint32_t w) { return lop3<(0xF0 & 0xCC) ^ 0xAA>(w, 0xF0F0F0F0u, 0x80808080u); }
__device__ __forceinline__ uint32_t q16_lo(uint32_t w) { return lop3<(0xF0 & 0xCC) ^ 0xAA>(w << 4, 0xF0F0F0F0u, 0x80808080u); }

// Eight consecutive activations as fp32 (16-byte aligned).
template <typename AT>
__device__ __forceinline__ void load8(const AT* p, float (&f)[8]) {
    if constexpr (sizeof(AT) == 4) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        const AT* e = reinterpret_cast<const AT*>(&v);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = to_f32(e[i]);
    }
}

// Activation pieces.  One CTA per scale group, 16 threads per token slot, 8
// consecutive k per thread.  Writes the pieces of token slots [0, slots) (zero
// beyond M), 2^-s of all 16 slots of the group and, with `sums`, the group's
// sum of x per slot.
//
// RES (fp32 activations): x keeps 30 bits as two fixed-point copies.  Slot m <
// slots/2 holds token m as above, x_hi = 2^-s round(2^s x); slot slots/2 + m
// holds the rest, x - x_hi (exact in fp32, |x - x_hi| <= 2^-s-1), in steps of
// 2^-(s+15).  Both slots of a token land in the same lanes (tiles j and
// j + NT/2), whose sums the GEMM adds before storing.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

template <typename AT, bool RES, bool T2 = false>
__global__ void __launch_bounds__(kPrepThreads) x_prep_kernel(const AT* __restrict__ A, int M, int K, int group,
                                                              int slots, int8_t* __restrict__ pieces,
                                                              float* __restrict__ xscale, float* __restrict__ xsum,
                                                              int* __restrict__ xkb) {
    if (threadIdx.x == 0) pdl_launch_dependents();
    // A may come from the previous kernel, and that kernel may still read the
    // pieces of the previous call.
    pdl_wait();
    const int gi = blockIdx.x;
    const int m = threadIdx.x >> 4, l16 = threadIdx.x & 15;
    const bool res = RES && m >= slots / 2 && m < slots;
    const int tok = res ? m - slots / 2 : m;  // the token whose values this slot holds
    const int oct = group / 8;
    const AT* row = A + (size_t)tok * K + (size_t)gi * group;
    float mx = 0.f, sum = 0.f;
    int bad = 0;
    if (tok < M) {
        for (int o = l16; o < oct; o += 16) {
            float f[8];
            load8(row + 8 * o, f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                bad |= !isfinite(f[i]);
                mx = fmaxf(mx, fabsf(f[i]));
                sum += f[i];
            }
        }
    }
#pragma unroll
    for (int d = 8; d >= 1; d >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
        sum += __shfl_xor_sync(0xffffffffu, sum, d);
        bad |= __shfl_xor_sync(0xffffffffu, bad, d);
    }
    // x * 2^s < 2^14 for every |x| <= mx, so |x_fixed| <= 2^14 and h = (x_fixed + 128) >> 8 <= 64;
    // the rest of a RES slot is below 2^-s-1, so (x - x_hi) * 2^(s+15) <= 2^14 as well.
    int s = 0;
    float xs = 0.f;
    if (bad) {
        xs = res ? 0.f : __int_as_float(0x7fc00000);
    } else if (mx > 0.f) {
        s = 13 - ilogbf(mx);
        xs = ldexpf(1.f, res ? -(s + 15) : -s);
    }
    if (l16 == 0) {
        xscale[(size_t)gi * 16 + m] = tok < M ? xs : 0.f;
        if (xsum) xsum[(size_t)gi * 16 + m] = (tok < M && !res) ? sum : 0.f;
    }
    if (m >= slots) return;
    for (int o = l16; o < oct; o += 16) {
        int xf[8];
        if (tok < M && !bad) {
            float f[8];
            load8(row + 8 * o, f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float hi = rintf(ldexpf(f[i], s));
                xf[i] = res ? (int)rintf(ldexpf(f[i] - ldexpf(hi, -s), s + 15)) : (int)hi;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) xf[i] = 0;
        }
        uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
        // int4: byte j of word A holds element {0,2,1,3}[j], of word B element {4,6,5,7}[j];
        // ternary: the elements in natural order (0..3, 4..7), interleaved with the other octet below
        constexpr int kOrder[8] = {0, 2, 1, 3, 4, 6, 5, 7};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int v = xf[T2 ? j : kOrder[j]];
            const int h = (v + 128) >> 8;
            const int l = v - (h << 8);
            hw[j >> 2] |= (uint32_t)(h & 0xFF) << (8 * (j & 3));
            lw[j >> 2] |= (uint32_t)(l & 0xFF) << (8 * (j & 3));
        }
        const int k0 = gi * group + 8 * o;
        const int kb = k0 >> 6, t = (k0 >> 4) & 3, hh = (k0 >> 3) & 1;
        int8_t* tile = pieces + (size_t)kb * slots * 128;
        uint32_t* ph = reinterpret_cast<uint32_t*>(tile + ((m * 2 + 0) * 4 + t) * 16);
        uint32_t* pl = reinterpret_cast<uint32_t*>(tile + ((m * 2 + 1) * 4 + t) * 16);
        if constexpr (T2) {
            // The 16 bytes of lane t are elements {0,8,1,9}, {2,10,3,11}, {4,12,5,13},
            // {6,14,7,15} of its 16 k: the order in which (w >> 2s) & 0x03030303 takes
            // codes out of a TILE_T2 word, so the kernel needs no byte permutes.  The
            // other octet of the 16 k is in the neighbouring lane (o ^ 1, as group % 64
            // == 0): the low-k lane writes words 0-1, the high-k lane words 2-3.
            const unsigned act = __activemask();
            const uint32_t rh = __shfl_xor_sync(act, hh ? hw[0] : hw[1], 1);
            const uint32_t rl = __shfl_xor_sync(act, hh ? lw[0] : lw[1], 1);
            if (!hh) {
                ph[0] = prmt(hw[0], rh, 0x5140u);
                ph[1] = prmt(hw[0], rh, 0x7362u);
                pl[0] = prmt(lw[0], rl, 0x5140u);
                pl[1] = prmt(lw[0], rl, 0x7362u);
            } else {
                ph[2] = prmt(rh, hw[1], 0x5140u);
                ph[3] = prmt(rh, hw[1], 0x7362u);
                pl[2] = prmt(rl, lw[1], 0x5140u);
                pl[3] = prmt(rl, lw[1], 0x7362u);
            }
        } else {
            ph[hh] = hw[0];
            ph[2 + hh] = hw[1];
            pl[hh] = lw[0];
            pl[2 + hh] = lw[1];
        }
        if (xkb) {  // ternary: sum of the fixed-point x over each k-block (8 octets = 8 lanes)
            int sum8 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) sum8 += xf[i];
            // the 8 lanes of an aligned octet group run this pass together (oct % 8 == 0)
            const unsigned act = __activemask();
#pragma unroll
            for (int d = 4; d >= 1; d >>= 1) sum8 += __shfl_xor_sync(act, sum8, d);
            if ((l16 & 7) == 0) xkb[(size_t)kb * 16 + m] = sum8;
        }
    }
}

// Ternary codes c = q + 1 (2 bits, TILE_T2 word of 16 consecutive k of one
// column, code e at field (e >> 1) + 8 (e & 1)) as u8 MMA operands: field class
// s (fields s, s + 4, s + 8, s + 12, one per byte) is (w >> 2s) & 0x03030303,
// i.e. codes e = {0,8,1,9} (s = 0), {2,10,3,11}, {4,12,5,13}, {6,14,7,15}; the
// prep kernel writes the ternary activation pieces in that order, so MMA 0
// takes classes 0 (slots 4t..) and 1 (slots 16 + 4t..) and MMA 1 classes 2, 3.
__device__ __forceinline__ void t2_operands(uint32_t w, uint32_t& m0a, uint32_t& m0b, uint32_t& m1a, uint32_t& m1b) {
    m0a = w & 0x03030303u;
    m0b = (w >> 2) & 0x03030303u;
    m1a = (w >> 4) & 0x03030303u;
    m1b = (w >> 6) & 0x03030303u;
}
// D (16x8 s32) += A (16x32 u8) x B (32x8 s8).
__device__ __forceinline__ void imma_16832_u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// RES: fp32 activations in two slots per token (x_prep_kernel); tiles j and
// j + NT/2 hold the two parts of the same tokens.
template <int NT, bool RES, int WB, typename ST, typename OT>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) decode_i8_kernel(const __grid_constant__ I8Params p) {
    using L = RingI8<NT, WB, ST>;
    constexpr int kStages = L::kStages;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    float2* pair_buf = reinterpret_cast<float2*>(ring + kStages * L::kBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * L::kBytes + L::kPair);
    uint64_t* empty = full + kStages;
    volatile int* s_last = reinterpret_cast<volatile int*>(empty + kStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WB);
    const int KB = geo.KB;
    const long long U = geo.units();
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    const long long u_begin = range_begin(U, G, c), u_end = range_begin(U, G, c + 1);
    const int upg = p.group / kBlockK;  // k-blocks per scale group
    // Scale group of a k-block: a shift for the usual power-of-two groups (64,
    // 128, 256), a division otherwise (the branch is uniform).
    const int upg_sh = (upg & (upg - 1)) == 0 ? __ffs(upg) - 1 : -1;
    auto grp = [upg, upg_sh](int kb) { return upg_sh >= 0 ? kb >> upg_sh : kb / upg; };

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1 + 32 * kProducerWarps);  // the bulk copy's expect-tx + one cp.async arrival per producer lane
            mbar_init(&empty[i], kNC);
        }
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        pdl_launch_dependents();
    }
    __syncthreads();

    if (warp >= kProducerWarp) {
        // --------------------------------------------------------- producers
        // A warp holding more than a few DRAM-latency cp.async per lane stalls
        // its issue; the producer warps share them so that none does.
        const int pl = (warp - kProducerWarp) * 32 + lane;  // producer lane 0 .. 32 * kProducerWarps - 1
        const uint64_t pol = l2_policy_evict_first();
        const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
        auto stage_ptr = [&](int it) { return ring + (it % kStages) * L::kBytes; };
        // Codes (one bulk copy) and weight-scale rows (16-byte cp.async spread over
        // the lanes) of stage `it`: no earlier kernel writes them.
        auto issue_w = [&](int it, const Span& d) {
            const int slot = it % kStages;
            uint8_t* st = stage_ptr(it);
            const int width = geo.width(d.sg);
            const int s_chunks = width * kStripCols * (int)sizeof(ST) / 16;  // 16-byte pieces of one scale row
            const uint32_t wbytes = (uint32_t)d.n * (uint32_t)width * (uint32_t)geo.CB;
            const int g_first = grp(d.kb), ng = grp(d.kb + d.n - 1) - g_first + 1;
            if (pl == 0) {
                mbar_arrive_expect_tx(&full[slot], wbytes);
                bulk_g2s_hint(st, p.W + geo.unit_offset((long long)d.sg * KB + d.kb), wbytes, &full[slot], pol);
            }
            for (int i = pl; i < ng * s_chunks; i += 32 * kProducerWarps) {
                const int r = i / s_chunks, cidx = i - r * s_chunks;
                const size_t off = (size_t)(g_first + r) * p.N + (size_t)d.sg * kGroupCols;
                cp_async16(st + L::kS + r * L::kSUnit + 16 * cidx, Sb + off * sizeof(ST) + 16 * cidx);
                if constexpr (L::kBias)
                    if (p.bias)
                        cp_async16(st + L::kB + r * L::kSUnit + 16 * cidx,
                                   reinterpret_cast<const uint8_t*>(p.bias) + off * 4 + 16 * cidx);
            }
        };
        // Activation pieces and their scales (written by the preceding kernel), then
        // every lane's arrival once its copies of the stage have landed.
        auto issue_x = [&](int it, const Span& d) {
            const int slot = it % kStages;
            uint8_t* st = stage_ptr(it);
            const int g_first = grp(d.kb), ng = grp(d.kb + d.n - 1) - g_first + 1;
            const int p_chunks = d.n * NT * kTileBytes / 16;
            const int8_t* psrc = p.pieces + (size_t)d.kb * NT * kTileBytes;
            for (int i = pl; i < p_chunks; i += 32 * kProducerWarps) cp_async16(st + L::kX + 16 * i, psrc + 16 * i);
            if constexpr (WB == 2)
                for (int i = pl; i < d.n * 4; i += 32 * kProducerWarps)
                    cp_async16(st + L::kXK + 16 * i, p.xkb + (size_t)d.kb * 16 + 4 * i);
            for (int i = pl; i < ng * 4; i += 32 * kProducerWarps) {
                cp_async16(st + L::kXS + 16 * i, p.xscale + (size_t)g_first * 16 + 4 * i);
                if constexpr (L::kBias)
                    if (p.bias) cp_async16(st + L::kXQ + 16 * i, p.xsum + (size_t)g_first * 16 + 4 * i);
            }
            cp_async_mbar_arrive(&full[slot]);
        };
        Walker wk(u_begin, u_end, KB, kUPS);
        Span d;
        Span pend[kStages];
        int it = 0;
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
        if (lane == 0)
            for (int j = it - kStages < 0 ? 0 : it - kStages; j < it; ++j)
                mbar_wait(&full[j % kStages], (uint32_t)(j / kStages) & 1u, p.err);
        __syncwarp();
        return;
    }

    // ------------------------------------------------------------ consumers
    // kHalves warps per strip: with two, half 0 takes the first half of every
    // stage's k-blocks and half 1 the rest, and their sums meet in shared
    // memory when a strip group is done.
    pdl_wait();
    const int g = lane >> 2, t = lane & 3;
    const int sl = warp & 7, half = warp >> 3;
    OT* C = reinterpret_cast<OT*>(p.C);
    float facc[NT][2];
    int iacc[NT][4];
    int csum[NT];  // ternary: sum of the fixed-point x over the k-blocks in iacc (per token)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        facc[j][0] = facc[j][1] = 0.f;
        csum[j] = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) iacc[j][i] = 0;
    }

    // Exact integer sums of one scale group -> fp32 (scale row gl of the stage).
    auto flush_ints = [&](const uint8_t* stage, int gl) {
        const int nl = sl * kStripCols + g;
        const uint8_t* sp = stage + L::kS + gl * L::kSUnit;
        const float s0 = to_f32(*reinterpret_cast<const ST*>(sp + nl * sizeof(ST)));
        const float s1 = to_f32(*reinterpret_cast<const ST*>(sp + (nl + 8) * sizeof(ST)));
        const float* xs = reinterpret_cast<const float*>(stage + L::kXS + gl * 64);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            // int4: the MMA saw 16 q, so 2^-s / 16; ternary: q + 1, so 2^-s and minus sum x
            const float f = xs[kTokTile * j + t] * (WB == 4 ? 0.0625f : 1.f);
            const int v0 = iacc[j][0] * 256 + iacc[j][1] - csum[j];
            const int v1 = iacc[j][2] * 256 + iacc[j][3] - csum[j];
            facc[j][0] = fmaf((float)v0, s0 * f, facc[j][0]);
            facc[j][1] = fmaf((float)v1, s1 * f, facc[j][1]);
            csum[j] = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) iacc[j][i] = 0;
        }
    };

    // Bias term of scale group gl of the stage, added once per group (at its first
    // k-block): w = u s + b = q s + (8 s + b) with q = u - 8, so
    // sum_k x_k w_k = s sum_k x_k q_k + (8 s + b) sum_k x_k.
    auto add_bias = [&](const uint8_t* stage, int gl) {
        if constexpr (L::kBias) {
            const int nl = sl * kStripCols + g;
            const float* sp = reinterpret_cast<const float*>(stage + L::kS + gl * L::kSUnit);
            const float* bp = reinterpret_cast<const float*>(stage + L::kB + gl * L::kSUnit);
            const float c0 = fmaf(8.f, sp[nl], bp[nl]), c1 = fmaf(8.f, sp[nl + 8], bp[nl + 8]);
            const float* xq = reinterpret_cast<const float*>(stage + L::kXQ + gl * 64);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const float xsj = xq[kTokTile * j + t];
                facc[j][0] = fmaf(xsj, c0, facc[j][0]);
                facc[j][1] = fmaf(xsj, c1, facc[j][1]);
            }
        }
    };

    auto store_pair = [&](int sg, int j, float v0, float v1) {
        const int n = sg * kGroupCols + sl * kStripCols + g;
        const int tok = kTokTile * j + t;
        if (tok < p.M) {
            C[(size_t)tok * p.N + n] = from_f32<OT>(v0);
            C[(size_t)tok * p.N + n + 8] = from_f32<OT>(v1);
        }
    };

    const int first_sg = (int)(u_begin / KB);
    int pend_sg[2] = {-1, -1};  // strip groups handed to the fixup, by slot
    int nflush = 0;
    // Strip group `sg` is done for this CTA: half 1 hands its sums to half 0,
    // which stores the group or, when other CTAs share it, writes the partial
    // and lets thread 0 count the arrival (the last arriver sums after the loop).
    auto flush_group = [&](int sg) {
        if constexpr (RES) {
#pragma unroll
            for (int j = 0; j < NT / 2; ++j) {
                facc[j][0] += facc[j + NT / 2][0];
                facc[j][1] += facc[j + NT / 2][1];
            }
        }
        if constexpr (kHalves > 1) {
            float2* xch = pair_buf + ((nflush & 1) * 8 + sl) * (NT * 32);
            ++nflush;
            if (half == 1) {
#pragma unroll
                for (int j = 0; j < NT; ++j) xch[j * 32 + lane] = make_float2(facc[j][0], facc[j][1]);
            }
            named_bar_sync(kPairBar, kNC * 32);
            if (half == 0) {
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const float2 v = xch[j * 32 + lane];
                    facc[j][0] += v.x;
                    facc[j][1] += v.y;
                }
            }
        }
        if (half == 0) {
            const int width = geo.width(sg);
            const long long g0 = (long long)sg * KB, g1 = g0 + KB;
            if (g0 >= u_begin && g1 <= u_end) {
                if (sl < width)
#pragma unroll
                    for (int j = 0; j < NT; ++j) store_pair(sg, j, facc[j][0], facc[j][1]);
            } else {
                const int slot = sg == first_sg ? 0 : 1;
                float2* mine = p.partials + (((size_t)c * 2 + slot) * 8 + sl) * (NT * 32);
#pragma unroll
                for (int j = 0; j < NT; ++j) mine[j * 32 + lane] = make_float2(facc[j][0], facc[j][1]);
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
        for (int j = 0; j < NT; ++j) facc[j][0] = facc[j][1] = 0.f;
    };

    bool waits_ok = true;
    Walker wk(u_begin, u_end, KB, kUPS);
    Span d;
    int it = 0, cur = -1;
    while (wk.next(d)) {
        if (d.sg != cur) {
            if (cur >= 0) flush_group(cur);
            cur = d.sg;
        }
        const int slot = it % kStages;
        if (waits_ok) waits_ok = mbar_wait(&full[slot], (uint32_t)(it / kStages) & 1u, p.err);
        const uint8_t* stage = ring + slot * L::kBytes;
        const int width = geo.width(d.sg);
        constexpr int kPer = kUPS / kHalves;  // k-blocks of a stage per warp of the strip
#pragma unroll
        for (int bb = 0; bb < kPer; bb += kBatch) {
        const int b0 = half * kPer + bb;  // this batch: k-blocks [b0, min(b0 + kBatch, n)) of the stage
        const int bn = d.n - b0 < kBatch ? d.n - b0 : kBatch;
        if (sl < width && bn > 0) {
            constexpr int kCBw = WB == 4 ? 512 : 256, kLaneB = WB == 4 ? 16 : 8;  // chunk and lane bytes
            const uint32_t unit_bytes = (uint32_t)width * kCBw;
            const uint8_t* wbase = stage + (b0 * (int)unit_bytes) + sl * kCBw + lane * kLaneB;
            const int g_stage = grp(d.kb);
            const int g_b0 = grp(d.kb + b0);
            int gl = g_b0 - g_stage;                     // scale row of k-block b0
            int gend = (g_b0 + 1) * upg - (d.kb + b0);  // k-blocks of the batch to its group's end
            uint4 wv[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if constexpr (WB == 4) {
                    wv[u] = u < bn ? *reinterpret_cast<const uint4*>(wbase + u * unit_bytes) : make_uint4(0u, 0u, 0u, 0u);
                } else {
                    const uint2 v = u < bn ? *reinterpret_cast<const uint2*>(wbase + u * unit_bytes) : make_uint2(0u, 0u);
                    wv[u] = make_uint4(v.x, v.y, 0u, 0u);
                }
            }
            const uint8_t* xbase = stage + L::kX + b0 * L::kXUnit + lane * 16;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if (u >= bn) break;
                if constexpr (L::kBias)
                    if (p.bias && grp(d.kb + b0 + u) * upg == d.kb + b0 + u) add_bias(stage, gl);
                // operands a0..a3 of MMA 0 (l*) and MMA 1 (h*): rows g / g + 8, k-slots 4t.. / 16 + 4t..
                uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
                if constexpr (WB == 4) {
                    l0 = q16_lo(wv[u].x), l1 = q16_lo(wv[u].z), l2 = q16_lo(wv[u].y), l3 = q16_lo(wv[u].w);
                    h0 = q16_hi(wv[u].x), h1 = q16_hi(wv[u].z), h2 = q16_hi(wv[u].y), h3 = q16_hi(wv[u].w);
                } else {
                    t2_operands(wv[u].x, l0, l2, h0, h2);  // column g
                    t2_operands(wv[u].y, l1, l3, h1, h3);  // column g + 8
                }
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint4 xv = *reinterpret_cast<const uint4*>(xbase + u * L::kXUnit + j * kTileBytes);
                    if constexpr (WB == 4) {
                        imma_16832(iacc[j], l0, l1, l2, l3, xv.x, xv.y);
                        imma_16832(iacc[j], h0, h1, h2, h3, xv.z, xv.w);
                    } else {
                        imma_16832_u8(iacc[j], l0, l1, l2, l3, xv.x, xv.y);
                        imma_16832_u8(iacc[j], h0, h1, h2, h3, xv.z, xv.w);
                        csum[j] += *reinterpret_cast<const int*>(stage + L::kXK + (b0 + u) * 64 + 4 * (kTokTile * j + t));
                    }
                }
                if (u + 1 == gend) {
                    flush_ints(stage, gl);
                    ++gl;
                    gend += upg;
                } else if (u + 1 == bn) {
                    flush_ints(stage, gl);
                }
            }
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
            float2 sum[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) sum[j] = make_float2(0.f, 0.f);
            // Up to kFix partials in flight at once (one L2 round trip per batch), summed
            // in CTA order.
            constexpr int kFix = NT <= 2 ? 8 : 4;
            for (int q0 = c_first; q0 <= c_last; q0 += kFix) {
                float2 v[kFix][NT];
#pragma unroll
                for (int i = 0; i < kFix; ++i) {
                    const int q = q0 + i;
                    if (q <= c_last) {
                        const int qslot = (int)(range_begin(U, G, q) / KB) == sg ? 0 : 1;
                        const float2* src = p.partials + (((size_t)q * 2 + qslot) * 8 + sl) * (NT * 32);
#pragma unroll
                        for (int j = 0; j < NT; ++j) v[i][j] = __ldcg(src + j * 32 + lane);
                    }
                }
#pragma unroll
                for (int i = 0; i < kFix; ++i)
                    if (q0 + i <= c_last)
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            sum[j].x += v[i][j].x;
                            sum[j].y += v[i][j].y;
                        }
            }
            if (sl < geo.width(sg))
#pragma unroll
                for (int j = 0; j < NT; ++j) store_pair(sg, j, sum[j].x, sum[j].y);
            if (threadIdx.x == 0) p.counters[sg] = 0u;
        }
    }
}

}  // namespace
}  // namespace hq

namespace hq {

namespace {

using I8Fn = void (*)(I8Params);

template <int NT, bool RES, typename ST, typename OT, int WB = 4>
std::pair<I8Fn, int> i8_kernel() {
    return {decode_i8_kernel<NT, RES, WB, ST, OT>, RingI8<NT, WB, ST>::kSmem};
}

template <typename ST, typename OT>
std::pair<I8Fn, int> pick_nt(int NT) {
    return NT == 1 ? i8_kernel<1, false, ST, OT>() : i8_kernel<2, false, ST, OT>();
}

template <typename ST>
std::pair<I8Fn, int> pick_out(DType c, int NT) {
    if (c == DType::F16) return pick_nt<ST, __half>(NT);
    if (c == DType::BF16) return pick_nt<ST, __nv_bfloat16>(NT);
    return pick_nt<ST, float>(NT);
}

// Tiles of 4 token slots the kernel runs: fp32 activations (M <= 4) take two,
// the token parts x_hi and x - x_hi.
int i8_tiles(const GemmArgs& a) { return a.a_dtype == DType::F32 ? 2 : (a.M + kTokTile - 1) / kTokTile; }

std::pair<I8Fn, int> select_i8(const GemmArgs& a) {
    if (a.wbits == 2) {  // ternary: 16-bit activations and scales of the same type, M <= 4
        if (a.s_dtype == DType::F16)
            return a.c_dtype == DType::F32 ? i8_kernel<1, false, __half, float, 2>()
                                           : i8_kernel<1, false, __half, __half, 2>();
        return a.c_dtype == DType::F32 ? i8_kernel<1, false, __nv_bfloat16, float, 2>()
                                       : i8_kernel<1, false, __nv_bfloat16, __nv_bfloat16, 2>();
    }
    if (a.a_dtype == DType::F32) {
        // fp32 activations: fp32 output (hq_gemm's rule c_dtype == a_dtype or f32)
        if (a.s_dtype == DType::F16) return i8_kernel<2, true, __half, float>();
        if (a.s_dtype == DType::BF16) return i8_kernel<2, true, __nv_bfloat16, float>();
        return i8_kernel<2, true, float, float>();
    }
    const int NT = i8_tiles(a);
    if (a.s_dtype == DType::F16) return pick_out<__half>(a.c_dtype, NT);
    if (a.s_dtype == DType::BF16) return pick_out<__nv_bfloat16>(a.c_dtype, NT);
    return pick_out<float>(a.c_dtype, NT);
}

size_t pieces_bytes(int K) { return (size_t)(K / kBlockK) * 4 * kTileBytes; }

size_t counters_bytes(int N) {
    const size_t nsg = (size_t)((N / kStripCols + kGroupStrips - 1) / kGroupStrips);
    return (nsg * 4 + 255) & ~(size_t)255;
}

int grid_ctas(int N, int K, int dev) {
    const long long U = TileGeom(K, N, 4).units();
    const long long G = (long long)device_info(dev).sm_count * kCtasPerSm;
    return (int)(U < G ? U : G);
}

// Counters, then two partial tiles per CTA (8 strips x 4 token tiles x 32 lanes x float2).
size_t split_bytes(int N, int K, int dev) {
    return counters_bytes(N) + (size_t)grid_ctas(N, K, dev) * 2 * 8 * 4 * 32 * sizeof(float2);
}
size_t xscale_bytes(int K) { return ((size_t)(K / kBlockK) * 64 + 255) & ~(size_t)255; }

}  // namespace

bool decode_i8_supported(const GemmArgs& a) {
    if (a.wbits == 2) {  // ternary: one tile of 4 token slots, 16-bit activations, scales of their type
        if (a.M < 1 || a.M > 4 || a.bias || (a.a_dtype != DType::F16 && a.a_dtype != DType::BF16)) return false;
        if (a.s_dtype != a.a_dtype || (a.c_dtype != a.a_dtype && a.c_dtype != DType::F32)) return false;
        return a.group % kBlockK == 0 && a.K % a.group == 0;
    }
    if (a.wbits != 4 || a.M < 1 || a.M > 8) return false;  // one or two tiles of 4 token slots
    if (a.a_dtype == DType::F32) {
        if (a.M > 4 || a.c_dtype != DType::F32) return false;
    } else if (a.a_dtype != DType::F16 && a.a_dtype != DType::BF16) {
        return false;
    }
    if (a.c_dtype != a.a_dtype && a.c_dtype != DType::F32) return false;
    // The reference form: fp32 scales and biases, with f16 or f32 activations (the same
    // combinations the cluster split-K kernel takes).
    if (a.bias && (a.s_dtype != DType::F32 || a.a_dtype == DType::BF16)) return false;
    return a.group % kBlockK == 0 && a.K % a.group == 0;
}

// split state, activation pieces, x scales, x sums per scale group, x sums per k-block (ternary)
size_t decode_i8_workspace_bytes(int N, int K, int dev) {
    return split_bytes(N, K, dev) + pieces_bytes(K) + 3 * xscale_bytes(K);
}

cudaError_t launch_decode_i8(const GemmArgs& a, bool early_weights) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t split = split_bytes(a.N, a.K, dev);
    if (!a.ws || a.ws_bytes < decode_i8_workspace_bytes(a.N, a.K, dev)) return cudaErrorInvalidValue;
    const int NT = i8_tiles(a);
    int8_t* pieces = reinterpret_cast<int8_t*>(a.ws + split);
    float* xscale = reinterpret_cast<float*>(a.ws + split + pieces_bytes(a.K));
    float* xsum = a.bias ? reinterpret_cast<float*>(a.ws + split + pieces_bytes(a.K) + xscale_bytes(a.K)) : nullptr;
    int* xkb = a.wbits == 2 ? reinterpret_cast<int*>(a.ws + split + pieces_bytes(a.K) + 2 * xscale_bytes(a.K))
                            : nullptr;

    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;

    // 1. activation pieces
    cudaLaunchConfig_t pc = {};
    pc.gridDim = dim3((unsigned)(a.K / a.group));
    pc.blockDim = dim3(kPrepThreads);
    pc.stream = a.stream;
    pc.attrs = pdl;
    pc.numAttrs = 1;
    const bool t2 = a.wbits == 2;
    if (a.a_dtype == DType::F16)
        e = cudaLaunchKernelEx(&pc, t2 ? x_prep_kernel<__half, false, true> : x_prep_kernel<__half, false>,
                               static_cast<const __half*>(a.A), a.M, a.K, a.group, NT * kTokTile, pieces, xscale,
                               xsum, xkb);
    else if (a.a_dtype == DType::BF16)
        e = cudaLaunchKernelEx(&pc, t2 ? x_prep_kernel<__nv_bfloat16, false, true> : x_prep_kernel<__nv_bfloat16, false>,
                               static_cast<const __nv_bfloat16*>(a.A), a.M, a.K, a.group, NT * kTokTile, pieces,
                               xscale, xsum, xkb);
    else
        e = cudaLaunchKernelEx(&pc, x_prep_kernel<float, true>, static_cast<const float*>(a.A), a.M, a.K, a.group,
                               NT * kTokTile, pieces, xscale, xsum, static_cast<int*>(nullptr));
    if (e != cudaSuccess) return e;

    // 2. the GEMM
    const std::pair<I8Fn, int> k = select_i8(a);
    e = ensure_smem_attr(reinterpret_cast<const void*>(k.first), dev, k.second);
    if (e != cudaSuccess) return e;
    I8Params p;
    memset(&p, 0, sizeof p);
    p.W = a.W;
    p.S = a.S;
    p.bias = a.bias;
    p.pieces = pieces;
    p.xscale = xscale;
    p.xsum = xsum;
    p.xkb = xkb;
    p.C = a.C;
    p.err = device_error_word(dev);
    p.counters = reinterpret_cast<unsigned*>(a.ws);
    p.partials = reinterpret_cast<float2*>(a.ws + counters_bytes(a.N));
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.group = a.group;
    p.early_weights = (early_weights && !a.weights_just_written) ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid_ctas(a.N, a.K, dev));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)k.second;
    cfg.stream = a.stream;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k.first, p);
}

}  // namespace hq
