// hq_prefill.cu -- tensor-core GEMM for M > 16 with the weights in tensor memory.
//
// The reference has no prefill GEMM (its decoder feeds the prompt one token at
// a time, hydrogen/src/model/native_decoder.cu:1297); this is the B200 kernel
// for the M >= 64 rows of the quantized linear layer.
//
// C^T tile = W_tile^T (128 output columns, tensor memory) x A_tile^T (256
// tokens, shared memory): the MMA's M side is one strip group of the weights,
// its N side the tokens.  The dequantised weights therefore go registers ->
// tensor memory (tcgen05.st) and never through shared memory, whose bandwidth
// the activation tiles (TMA in, MMA out) already use.
//   warp 8      producer: per 64-k block, one TMA box of activations (64 k x
//               256 tokens, 128-byte swizzle, rows >= M zero), the strip
//               group's packed codes (one bulk copy of the tile order) and the
//               group's scale row, into a 6-stage ring;
//   warps 0-7   dequantisers, two sets of four alternating k-blocks; warp q of
//               a set owns TMEM lanes [32q, 32q+32) = output columns: a thread
//               gathers its column's 64 codes (four 8-byte loads from a rotated
//               start lane: no bank conflicts), makes exact
//               q, multiplies by the group scale (rounded to the activation
//               type, as the tensor-core operand must be) and stores 32 packed
//               pairs to an 8-deep ring of A buffers in tensor memory; after a
//               tile's last k-block the same warps drain the accumulator
//               (tcgen05.ld) and store C, set h taking tokens [128h, 128h+128);
//   warp 9      one thread issues tcgen05.mma (M=128, N=256, K=16, A from
//               tensor memory, fp32 accumulate in 256 TMEM columns) and
//               commits completions; the warp owns the 512-column allocation.
// Tiles (strip group x 256 tokens) are walked persistently, token tile
// fastest, so the CTAs in flight share each strip group's codes through L2.
// Every wait is bounded (hq_common.cuh); nothing is allocated.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"
#include "hq_tmap.h"

#include <algorithm>
#include <cstring>
#include <type_traits>

namespace hq {

namespace {

constexpr int TM = 128;  // output columns per tile (MMA M)
constexpr int TN = 256;  // tokens per tile (MMA N)
constexpr int BK = 64;
constexpr int kStages = 6;
constexpr int kABufs = 8;
constexpr int kDqWarps = 8;
constexpr int kProdWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColD = 0;    // accumulator: 256 columns
constexpr uint32_t kColA = 256;  // A ring: kColA + 32 * buf

constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// kF32S: f32 scale rows (int4 only): per k-block the scale rows of its two
// 32-k halves, then their bias rows (any group of 32 or a multiple of 64).
template <int WBITS, bool kF32S = false>
struct TsLayout {
    static constexpr int kCB = WBITS == 4 ? 512 : 256;
    static constexpr int kX = TN * BK * 2;                 // activation tile, 1024-aligned at stage start
    static constexpr int kCodes = kGroupStrips * kCB;      // one strip group x 64 k
    static constexpr int kScale = kF32S ? 4 * TM * 4 : TM * 2;
    static constexpr int kStage = align_up(kX + kCodes + kScale, 1024);
    static constexpr int kStages = kF32S ? 5 : hq::kStages;  // six 38 KB stages exceed 227 KB
    static constexpr int kRing = kStages * kStage;
    static constexpr int kSmem = kRing + 256 + 1024;      // barriers + TMEM slot + alignment slack
};

struct alignas(64) PrefillTsParams {
    CUtensorMap x_map;  // [M][K] 16-bit: box 64 x 256, 128B swizzle, rows >= M read zero
    const uint8_t* W;
    const void* S;
    const float* bias;  // f32-scale kernels only; nullable (then w = (u - 8) s)
    void* C;
    unsigned* err;
    int M, N, K, group;
    int m_tiles, n_tiles;
};

template <bool kBF16>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t s) {
    return kBF16 ? bf16x2_mul(a, s) : hmul2_bits(a, s);
}

template <typename OT>
__device__ __forceinline__ OT cvt_out(float v) {
    return from_f32<OT>(v);
}

// f32-scale form of one tile word: its k pairs (e0,e1) (e2,e3) (e4,e5) (e6,e7)
// as u * s + b in fp32, rounded once to the operand type (fp32x2 arithmetic).
// fp16 operands take u exactly as fp16 pairs from the shared dequantiser and
// widen them on the FMA pipe.  bf16 operands OR each code field into the
// mantissa of 2^23 (2^23 + u; a high-nibble field in place reads 2^23 + 16 u and
// takes the exact scale s / 16), and one packed subtract gives the code.
template <bool kBF16>
__device__ __forceinline__ void affine_word(uint32_t w, float s, float b, uint32_t (&r)[4]) {
    unsigned long long bb, ss;
    asm("mov.b64 %0, {%1, %1};" : "=l"(bb) : "f"(b));
    asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
    if constexpr (!kBF16) {
        uint32_t uh[4];
        dequant_u4_f16<true>(w, uh);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const float2 u2 = __half22float2(*reinterpret_cast<const __half2*>(&uh[p]));
            unsigned long long v;
            asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(u2.x), "f"(u2.y));
            asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(v) : "l"(ss), "l"(bb));
            float x, y;
            asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v));
            __half2 h = __floats2half2_rn(x, y);
            r[p] = *reinterpret_cast<uint32_t*>(&h);
        }
    } else {
        constexpr uint32_t kM = 0x4B000000u;  // 2^23
        const uint32_t w8 = w >> 8, w16 = w >> 16, w24 = w >> 24;
        const uint32_t lo[4] = {(w & 0xFu) | kM, (w8 & 0xFu) | kM, (w & 0xF0u) | kM, (w8 & 0xF0u) | kM};
        const uint32_t hi[4] = {(w16 & 0xFu) | kM, (w24 & 0xFu) | kM, (w16 & 0xF0u) | kM, (w24 & 0xF0u) | kM};
        const float s16 = s * 0.0625f;
        unsigned long long mm, s16s;
        asm("mov.b64 %0, {%1, %1};" : "=l"(mm) : "r"(kM));
        asm("mov.b64 %0, {%1, %1};" : "=l"(s16s) : "f"(s16));
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            unsigned long long v;
            asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(lo[p]), "r"(hi[p]));
            asm("sub.f32x2 %0, %0, %1;" : "+l"(v) : "l"(mm));
            asm("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(v) : "l"(p < 2 ? ss : s16s), "l"(bb));
            float x, y;
            asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v));
            __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
            r[p] = *reinterpret_cast<uint32_t*>(&h);
        }
    }
}

template <int WBITS, typename T, typename OT, bool kF32S>
__global__ void __launch_bounds__(kThreads, 1) prefill_ts_kernel(const __grid_constant__ PrefillTsParams p) {
    using L = TsLayout<WBITS, kF32S>;
    constexpr int kStages = L::kStages;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr int kCB = L::kCB;
    constexpr uint32_t kIdesc = umma_idesc_f16(kBF16, TM, TN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + L::kRing);
    uint64_t* empty = full + kStages;
    uint64_t* a_full = empty + kStages;
    uint64_t* a_empty = a_full + kABufs;
    uint64_t* acc_full = a_empty + kABufs;
    uint64_t* acc_empty = acc_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileGeom geo(p.K, p.N, WBITS);
    const int KB = geo.KB;
    const int num_tiles = p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kABufs; ++i) {
            mbar_init(&a_full[i], 4);  // the four warps of the set that expanded this k-block
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kDqWarps);
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_last();  // codes are re-read by every token tile
            const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
            bool ok = true;
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int mt = tile % p.m_tiles, sg = tile / p.m_tiles;
                const int width = geo.width(sg);
                const uint32_t unit_bytes = (uint32_t)width * kCB;
                const uint32_t s_bytes = (uint32_t)width * kStripCols * (kF32S ? 4 : 2);
                const uint32_t srows = kF32S ? (p.bias ? 4u : 2u) : 1u;
                const size_t off = geo.unit_offset((long long)sg * KB);
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int slot = it % kStages;
                    if (ok) ok = mbar_wait(&empty[slot], ((uint32_t)(it / kStages) & 1u) ^ 1u, p.err);
                    uint8_t* st = ring + slot * L::kStage;
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)L::kX + unit_bytes + srows * s_bytes);
                    tma_load_2d(st, &p.x_map, kb * BK, mt * TN, &full[slot]);
                    bulk_g2s_hint(st + L::kX, p.W + off + (size_t)kb * unit_bytes, unit_bytes, &full[slot], pol);
                    if constexpr (kF32S) {
                        // rows of the block's two 32-k halves (the same row twice when group >= 64)
                        const uint8_t* Bb = reinterpret_cast<const uint8_t*>(p.bias);
                        for (int h = 0; h < 2; ++h) {
                            const size_t o = ((size_t)((kb * BK + 32 * h) / p.group) * p.N + (size_t)sg * TM) * 4;
                            bulk_g2s(st + L::kX + L::kCodes + h * TM * 4, Sb + o, s_bytes, &full[slot]);
                            if (Bb) bulk_g2s(st + L::kX + L::kCodes + (2 + h) * TM * 4, Bb + o, s_bytes, &full[slot]);
                        }
                    } else {
                        const int gi = kb * BK / p.group;
                        bulk_g2s(st + L::kX + L::kCodes, Sb + ((size_t)gi * p.N + (size_t)sg * TM) * 2, s_bytes,
                                 &full[slot]);
                    }
                }
            }
            // Copies still in flight land before the CTA exits.
            for (int j = it - kStages < 0 ? 0 : it - kStages; j < it; ++j)
                mbar_wait(&full[j % kStages], (uint32_t)(j / kStages) & 1u, p.err);
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ----------------------------------------------------------------- MMA
        if (lane == 0) {
            bool ok = true;
            int it = 0, tc = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
                if (ok) ok = mbar_wait(acc_empty, ((uint32_t)tc & 1u) ^ 1u, p.err);
                tc_fence_after();
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int ab = it % kABufs, slot = it % kStages;
                    // a_full implies full: the dequant warps saw the stage land first.
                    if (ok) ok = mbar_wait(&a_full[ab], (uint32_t)(it / kABufs) & 1u, p.err);
                    tc_fence_after();
                    const uint32_t xs = smem_u32(ring + slot * L::kStage);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_ts_f16(tmem + kColD, tmem + kColA + 32u * ab + 8u * k, sw128_kmajor_desc(xs + 32 * k),
                                    kIdesc, (kb | k) != 0);
                    umma_commit(&a_empty[ab]);
                    umma_commit(&empty[slot]);
                }
                umma_commit(acc_full);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------- dequant + epilogue
        const int set = warp >> 2, q = warp & 3;
        const int cl = 32 * q + lane;  // column within the strip group = TMEM lane
        const int sl = cl >> 4;        // strip
        const int c = lane & 15, g = c & 7, hh = c >> 3;
        const int rot = WBITS == 4 ? (g >> 1) : ((g >> 2) + 2 * (lane >> 4));  // bank-conflict-free gather
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        OT* C = reinterpret_cast<OT*>(p.C);
        bool ok = true;
        int it = 0, tc = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tc) {
            const int mt = tile % p.m_tiles, sg = tile / p.m_tiles;
            const int width = geo.width(sg);
            const bool valid = sl < width;
            for (int kb = 0; kb < KB; ++kb, ++it) {
                if ((it & 1) != set) continue;
                const int slot = it % kStages, ab = it % kABufs;
                if (ok) ok = mbar_wait(&full[slot], (uint32_t)(it / kStages) & 1u, p.err);
                if (ok) ok = mbar_wait(&a_empty[ab], ((uint32_t)(it / kABufs) & 1u) ^ 1u, p.err);
                __syncwarp();
                tc_fence_after();
                const uint8_t* st = ring + slot * L::kStage;
                const uint8_t* codes = st + L::kX + sl * kCB;
                uint32_t s2 = 0u;
                float sv[2] = {0.f, 0.f}, bv[2] = {0.f, 0.f};  // f32 form: per 32-k half
                if (valid) {
                    if constexpr (kF32S) {
                        const float* sr = reinterpret_cast<const float*>(st + L::kX + L::kCodes);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            sv[h] = sr[h * TM + cl];
                            bv[h] = p.bias ? sr[(2 + h) * TM + cl] : -8.f * sv[h];
                        }
                    } else {
                        const uint32_t v = *reinterpret_cast<const uint16_t*>(st + L::kX + L::kCodes + 2 * cl);
                        s2 = v | (v << 16);
                    }
                }
                const uint32_t ta = tmem + lane_base + kColA + 32u * ab;
                uint32_t cw[WBITS == 4 ? 8 : 4];  // this column's codes, k order
                if constexpr (WBITS == 4) gather_column_u4(codes, g, hh, rot, valid, cw);
                else gather_column_t2(codes, g, hh, rot, valid, cw);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    uint32_t r[8];
                    if constexpr (kF32S) {
                        // k 16t .. 16t+15 lie in the block's 32-k half t / 2
                        // the two words of k 16t .. 16t+15: TILE_U4 has them as lane t's
                        // pair; TILE_U4_K32 (group 32) as the first (t < 2) or second word
                        // of lanes 2(t % 2) and 2(t % 2) + 1
                        const bool k32 = p.group == 32;
                        const uint32_t w0 = k32 ? cw[4 * (t & 1) + (t >> 1)] : cw[2 * t];
                        const uint32_t w1 = k32 ? cw[4 * (t & 1) + 2 + (t >> 1)] : cw[2 * t + 1];
                        const float s = sv[t >> 1], b = bv[t >> 1];
                        uint32_t lo[4], hi[4];
                        affine_word<kBF16>(w0, s, b, lo);
                        affine_word<kBF16>(w1, s, b, hi);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            r[e] = lo[e];
                            r[4 + e] = hi[e];
                        }
                    } else if constexpr (WBITS == 4) {
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
                            r[e] = mul2<kBF16>(lo[e], s2);
                            r[4 + e] = mul2<kBF16>(hi[e], s2);
                        }
                    } else {
                        const uint32_t w = cw[t];
#pragma unroll
                        for (int e = 0; e < 8; ++e) r[e] = mul2<kBF16>(dequant_t2_pair<kBF16>(w, e), s2);
                    }
                    tmem_st8(ta + 8u * t, r);  // k = 16t .. 16t+15 of this k-block
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[ab]);
            }
            // Epilogue of this tile: tokens [128 set, 128 set + 128) of column cl.
            if (ok) ok = mbar_wait(acc_full, (uint32_t)tc & 1u, p.err);
            __syncwarp();
            tc_fence_after();
            const int col = sg * TM + cl;
            const bool col_ok = valid;
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_base + kColD + 128u * set + 32u * j, v);
                tmem_ld_wait();
                const int tok0 = mt * TN + 128 * set + 32 * j;
                if (col_ok) {
#pragma unroll
                    for (int r = 0; r < 32; ++r)
                        if (tok0 + r < p.M) C[(size_t)(tok0 + r) * p.N + col] = cvt_out<OT>(__uint_as_float(v[r]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------ CTA pairs
// The same tile pipeline over a cluster of two CTAs (cta_group::2): a pair
// tile is two strip groups (256 output columns) x 256 tokens.  Rank r
// dequantises strip group 2 p + r into its own tensor memory (rows r*128 ..
// of the M = 256 A operand and of the accumulator) and loads tokens
// [128 r, 128 r + 128) of the activation tile into its own shared memory (half
// of the B operand), so each SM reads half the activation bytes of the
// one-CTA kernel.  Rank 0's MMA thread issues M = 256 x N = 256 x K = 16 MMAs
// and commits every completion to the barrier at the same offset in both CTAs.
// The pipeline moves in units of two k-blocks (128 k): the MMA thread waits
// once and commits twice per eight MMAs (per-operation costs of the issuing
// thread -- ~140 cycles per completed wait, ~100 per MMA issue -- otherwise
// bound it).  Rank 1's dequant and epilogue warps arrive on rank 0's a_full /
// acc_empty; both ranks' activation loads count their bytes on rank 0's bfull,
// which rank 0's dequant warps wait for, so a_full alone releases the MMAs.
// Needs an even number of k-blocks (K % 128 == 0).
constexpr int kStagesPair = 5;  // stages of one unit
constexpr int kABufsPair = 4;   // A buffers of one unit (64 tensor-memory columns each)

template <int WBITS>
struct PairLayout {
    static constexpr int kCB = WBITS == 4 ? 512 : 256;
    static constexpr int kXB = (TN / 2) * BK * 2;          // this CTA's half tile of one k-block (16 KB)
    static constexpr int kX = 2 * kXB;
    static constexpr int kCodes = 2 * kGroupStrips * kCB;  // one strip group x 128 k
    static constexpr int kScale = 2 * TM * 2;              // up to two scale rows
    static constexpr int kStage = align_up(kX + kCodes + kScale, 1024);
    static constexpr int kRing = kStagesPair * kStage;
    static constexpr int kSmem = kRing + 512 + 1024;       // barriers + TMEM slot + alignment slack
};

template <int WBITS, typename T, typename OT>
__global__ void __launch_bounds__(kThreads, 1) prefill_pair_kernel(const __grid_constant__ PrefillTsParams p) {
    using L = PairLayout<WBITS>;
    constexpr int kS = kStagesPair, kAB = kABufsPair;
    constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr int kCB = L::kCB;
    constexpr uint32_t kIdesc = umma_idesc_f16(kBF16, 2 * TM, TN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + L::kRing);  // this CTA's codes + scales
    uint64_t* bfull = full + kS;                                    // rank 0: both activation halves
    uint64_t* empty = bfull + kS;
    uint64_t* a_full = empty + kS;  // rank 0: both ranks' dequant sets
    uint64_t* a_empty = a_full + kAB;
    uint64_t* acc_full = a_empty + kAB;
    uint64_t* acc_empty = acc_full + 1;  // rank 0: both ranks' epilogues
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const TileGeom geo(p.K, p.N, WBITS);
    const int KB = geo.KB, KU = KB / 2;
    const int pair_sgs = (geo.NSG + 1) / 2;
    const int num_tiles = p.m_tiles * pair_sgs;
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&bfull[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kAB; ++i) {
            mbar_init(&a_full[i], 8);  // four dequant warps of the set in each rank
            mbar_init(&a_empty[i], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * kDqWarps);
        fence_mbarrier_init();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both ranks' barriers and the allocation exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProdWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_last();  // codes are re-read by every token tile
            const uint8_t* Sb = reinterpret_cast<const uint8_t*>(p.S);
            bool ok = true;
            int it = 0;
            for (int tile = pair; tile < num_tiles; tile += npairs) {
                const int mt = tile % p.m_tiles, sg = 2 * (tile / p.m_tiles) + (int)rank;
                const int width = sg < geo.NSG ? geo.width(sg) : 0;
                const uint32_t unit_bytes = (uint32_t)width * kCB;
                const uint32_t s_bytes = (uint32_t)width * kStripCols * 2;
                const size_t off = width ? geo.unit_offset((long long)sg * KB) : 0;
                for (int u = 0; u < KU; ++u, ++it) {
                    const int slot = it % kS;
                    if (ok) ok = mbar_wait(&empty[slot], ((uint32_t)(it / kS) & 1u) ^ 1u, p.err);
                    uint8_t* st = ring + slot * L::kStage;
                    const int g0 = 2 * u * BK / p.group, g1 = (2 * u + 1) * BK / p.group;
                    const uint32_t rows = g1 != g0 ? 2u : 1u;
                    mbar_arrive_expect_tx(&full[slot], 2u * unit_bytes + rows * s_bytes);
                    if (width) {
                        bulk_g2s_hint(st + L::kX, p.W + off + (size_t)(2 * u) * unit_bytes, 2u * unit_bytes,
                                      &full[slot], pol);
                        for (uint32_t r = 0; r < rows; ++r)
                            bulk_g2s(st + L::kX + L::kCodes + r * TM * 2,
                                     Sb + ((size_t)(g0 + (int)r) * p.N + (size_t)sg * TM) * 2, s_bytes, &full[slot]);
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&bfull[slot], 2u * (uint32_t)L::kX);
                    const uint32_t bb = mapa_shared(smem_u32(&bfull[slot]), 0);
                    for (int h = 0; h < 2; ++h)
                        tma_load_2d_pair(st + h * L::kXB, &p.x_map, (2 * u + h) * BK, mt * TN + (TN / 2) * (int)rank,
                                         bb);
                }
            }
            // Every stage filled here has been consumed (its commit has landed) before exit.
            for (int j = it - kS < 0 ? 0 : it - kS; j < it; ++j)
                mbar_wait(&empty[j % kS], (uint32_t)(j / kS) & 1u, p.err);
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------- MMA (rank 0)
        if (lane == 0 && rank == 0) {
            bool ok = true;
            int it = 0, tc = 0;
            for (int tile = pair; tile < num_tiles; tile += npairs, ++tc) {
                if (ok) ok = mbar_wait(acc_empty, ((uint32_t)tc & 1u) ^ 1u, p.err);
                tc_fence_after();
                for (int u = 0; u < KU; ++u, ++it) {
                    const int ab = it % kAB, slot = it % kS;
                    // a_full implies both activation halves landed: rank 0's dequant warps
                    // waited on bfull before arriving.
                    if (ok) ok = mbar_wait(&a_full[ab], (uint32_t)(it / kAB) & 1u, p.err);
                    tc_fence_after();
                    const uint32_t xs = smem_u32(ring + slot * L::kStage);
#pragma unroll
                    for (int k = 0; k < 2 * BK / 16; ++k)
                        umma_ts_f16_pair(tmem + kColD, tmem + kColA + 64u * ab + 8u * k,
                                         sw128_kmajor_desc(xs + (k >> 2) * L::kXB + 32 * (k & 3)), kIdesc,
                                         (u | k) != 0);
                    umma_commit_pair(&a_empty[ab], 0x3);
                    umma_commit_pair(&empty[slot], 0x3);
                }
                umma_commit_pair(acc_full, 0x3);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------- dequant + epilogue
        const int set = warp >> 2, q = warp & 3;
        const int cl = 32 * q + lane;  // column within the strip group = TMEM lane
        const int sl = cl >> 4;        // strip
        const int c = lane & 15, g = c & 7, hh = c >> 3;
        const int rot = WBITS == 4 ? (g >> 1) : ((g >> 2) + 2 * (lane >> 4));  // bank-conflict-free gather
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        OT* C = reinterpret_cast<OT*>(p.C);
        bool ok = true;
        int it = 0, tc = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs, ++tc) {
            const int mt = tile % p.m_tiles, sg = 2 * (tile / p.m_tiles) + (int)rank;
            const int width = sg < geo.NSG ? geo.width(sg) : 0;
            const bool valid = sl < width;
            const uint32_t unit_bytes = (uint32_t)width * kCB;
            for (int u = 0; u < KU; ++u, ++it) {
                if ((it & 1) != set) continue;
                const int slot = it % kS, ab = it % kAB;
                if (ok) ok = mbar_wait(&full[slot], (uint32_t)(it / kS) & 1u, p.err);
                if (rank == 0 && ok) ok = mbar_wait(&bfull[slot], (uint32_t)(it / kS) & 1u, p.err);
                if (ok) ok = mbar_wait(&a_empty[ab], ((uint32_t)(it / kAB) & 1u) ^ 1u, p.err);
                __syncwarp();
                tc_fence_after();
                const uint8_t* st = ring + slot * L::kStage;
                const uint32_t ta = tmem + lane_base + kColA + 64u * ab;
                const int g0 = 2 * u * BK / p.group;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint8_t* codes = st + L::kX + h * unit_bytes + sl * kCB;
                    const int row = (2 * u + h) * BK / p.group - g0;
                    uint32_t s2 = 0u;
                    if (valid) {
                        const uint32_t v =
                            *reinterpret_cast<const uint16_t*>(st + L::kX + L::kCodes + row * TM * 2 + 2 * cl);
                        s2 = v | (v << 16);
                    }
                    uint32_t cw[WBITS == 4 ? 8 : 4];  // this column's codes, k order
                    if constexpr (WBITS == 4) gather_column_u4(codes, g, hh, rot, valid, cw);
                    else gather_column_t2(codes, g, hh, rot, valid, cw);
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
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
                                r[e] = mul2<kBF16>(lo[e], s2);
                                r[4 + e] = mul2<kBF16>(hi[e], s2);
                            }
                        } else {
                            const uint32_t w = cw[t];
#pragma unroll
                            for (int e = 0; e < 8; ++e) r[e] = mul2<kBF16>(dequant_t2_pair<kBF16>(w, e), s2);
                        }
                        tmem_st8(ta + 32u * h + 8u * t, r);  // k = 64h + 16t .. +15 of this unit
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(&a_full[ab]);
                    else mbar_arrive_cluster(&a_full[ab], 0);
                }
            }
            // Epilogue: this rank's 128 columns, tokens [128 set, 128 set + 128) of the tile.
            if (ok) ok = mbar_wait(acc_full, (uint32_t)tc & 1u, p.err);
            __syncwarp();
            tc_fence_after();
            const int col = sg * TM + cl;
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_base + kColD + 128u * set + 32u * j, v);
                tmem_ld_wait();
                const int tok0 = mt * TN + 128 * set + 32 * j;
                if (valid) {
#pragma unroll
                    for (int r = 0; r < 32; ++r)
                        if (tok0 + r < p.M) C[(size_t)(tok0 + r) * p.N + col] = cvt_out<OT>(__uint_as_float(v[r]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rank == 0) mbar_arrive(acc_empty);
                else mbar_arrive_cluster(acc_empty, 0);
            }
        }
    }

    tc_fence_before();
    cluster_sync();  // the pair's MMAs are complete and no arrive targets either CTA any more
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTmemCols);
    }
}

using PrefillTsFn = void (*)(PrefillTsParams);

template <int WBITS, typename T, bool PAIR>
PrefillTsFn ts_pick_out(DType c) {
    if (c == DType::F32) return PAIR ? prefill_pair_kernel<WBITS, T, float> : prefill_ts_kernel<WBITS, T, float, false>;
    if ((std::is_same<T, __half>::value && c == DType::F16) || (std::is_same<T, __nv_bfloat16>::value && c == DType::BF16))
        return PAIR ? prefill_pair_kernel<WBITS, T, T> : prefill_ts_kernel<WBITS, T, T, false>;
    return nullptr;
}

// f32 scale rows (int4, one-CTA kernel): group 32 or a multiple of 64; with a
// bias for fp16 activations, without one for bf16 (as the decode kernels).
template <typename T>
PrefillTsFn ts_pick_f32s(DType c) {
    if (c == DType::F32) return prefill_ts_kernel<4, T, float, true>;
    if ((std::is_same<T, __half>::value && c == DType::F16) || (std::is_same<T, __nv_bfloat16>::value && c == DType::BF16))
        return prefill_ts_kernel<4, T, T, true>;
    return nullptr;
}

template <bool PAIR>
PrefillTsFn ts_select(const GemmArgs& a) {
    if (!PAIR && a.wbits == 4 && a.s_dtype == DType::F32 && (a.group == 32 || a.group % BK == 0)) {
        if (a.a_dtype == DType::F16) return ts_pick_f32s<__half>(a.c_dtype);
        if (a.a_dtype == DType::BF16 && !a.bias) return ts_pick_f32s<__nv_bfloat16>(a.c_dtype);
        return nullptr;
    }
    if (a.bias || a.s_dtype != a.a_dtype || a.group % BK) return nullptr;
    if (a.a_dtype == DType::F16)
        return a.wbits == 4 ? ts_pick_out<4, __half, PAIR>(a.c_dtype) : ts_pick_out<2, __half, PAIR>(a.c_dtype);
    if (a.a_dtype == DType::BF16)
        return a.wbits == 4 ? ts_pick_out<4, __nv_bfloat16, PAIR>(a.c_dtype)
                            : ts_pick_out<2, __nv_bfloat16, PAIR>(a.c_dtype);
    return nullptr;
}

}  // namespace

size_t prefill_workspace_bytes(int, int, int, int, int) { return 0; }

bool prefill_supported(const GemmArgs& a) { return ts_select<false>(a) != nullptr; }

// CTA pairs (prefill_pair_kernel) unless the build sets HQ_PREFILL_PAIR=0.
#ifndef HQ_PREFILL_PAIR
#define HQ_PREFILL_PAIR 1
#endif

cudaError_t launch_prefill(const GemmArgs& a) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool pair = HQ_PREFILL_PAIR != 0 && a.K % (2 * BK) == 0 && ts_select<true>(a) != nullptr;
    const bool f32s = a.s_dtype == DType::F32;
    PrefillTsFn fn = pair ? ts_select<true>(a) : ts_select<false>(a);
    if (!fn) return cudaErrorInvalidValue;
    const int smem = pair ? (a.wbits == 4 ? PairLayout<4>::kSmem : PairLayout<2>::kSmem)
                          : (f32s ? TsLayout<4, true>::kSmem : a.wbits == 4 ? TsLayout<4>::kSmem : TsLayout<2>::kSmem);
    e = ensure_smem_attr(reinterpret_cast<const void*>(fn), dev, smem);
    if (e != cudaSuccess) return e;
    PrefillTsParams p;
    memset(&p, 0, sizeof p);
    // [M][K] 16-bit activations; a box is 64 k x 256 tokens (128 per CTA of a pair).
    e = make_tmap_2d(&p.x_map, a.A, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2,
                     BK, pair ? TN / 2 : TN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    p.W = a.W;
    p.S = a.S;
    p.bias = a.bias;
    p.C = a.C;
    p.err = device_error_word(dev);
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.group = a.group;
    p.m_tiles = (a.M + TN - 1) / TN;
    p.n_tiles = TileGeom(a.K, a.N, a.wbits).NSG;
    const int sms = device_info(dev).sm_count;
    if (!pair) {
        const int grid = std::min(p.m_tiles * p.n_tiles, sms);
        fn<<<grid, kThreads, smem, a.stream>>>(p);
        return cudaGetLastError();
    }
    // One pair per two SMs, capped by the pairs the GPU can hold at once (every
    // pair is persistent: a pair that waited for another to finish would idle).
    const int pair_tiles = p.m_tiles * ((p.n_tiles + 1) / 2);
    int pairs = std::min(pair_tiles, sms / 2);
    const int resident = max_active_clusters(reinterpret_cast<const void*>(fn), kThreads, smem, 2, dev);
    if (resident > 0) pairs = std::min(pairs, resident);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fn, p);
}

}  // namespace hq
