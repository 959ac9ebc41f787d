// hq_tq1.cu -- TQ1_0 (the reference's base-3 ternary block) kernels.
//
// TQ1_0 block (hydrogen/src/model/native_decoder.cu:32-36): fp16 d, packed[52]
// (bytes 0..49 hold 5 trits, bytes 50..51 hold 3, least significant first,
// trit = digit - 1), 2 pad bytes = 56 bytes per 256 weights; rows of
// in_dim/256 blocks.
//
// * tq1_0_gemv: drop-in for kernel_gemv_tq1_0 (:155-206) at M = 1 with fp32 x.
//   Two kernels behind one entry point:
//   - tq1_0_gemv_imma_kernel (in_dim % 1024 == 0, tables fit in shared memory):
//     the digits go to the integer tensor cores.  x is split exactly into four
//     int8 pieces of a 28-bit fixed-point copy (scale 2^(e-27), e = exponent of
//     max|x|); a byte's five base-3 digits come from a lane-replicated table
//     (one conflict-free 32-bit shared load per byte) as unsigned int8 lanes;
//     mma.sync m16n8k32 u8 x s8 -> s32 sums digit * piece for 16 rows, the
//     eight columns being (block parity) x (piece).  sum (digit - 1) * q =
//     sum digit * q - sum q, the second term a per-block constant; each block's
//     integer sums are scaled by the block's d when the block ends.  Integer
//     sums are exact: the only rounding is x's 28-bit fixed point and the fp32
//     combination of the per-block sums.
//   - tq1_0_gemv_kernel (every other shape, and any x holding NaN/Inf): one
//     warp per output row, each lane loads 8 contiguous bytes of the row (4
//     blocks per warp pass), x staged once per CTA in shared memory, byte ->
//     digits through a shared 256-entry table.
//   Both compute every row (unlike the reference launch at :1090-1091).
// * tq1_0_to_tile_t2: offline conversion into this library's 2-bit tile order
//   so that the fast decode / tensor-core kernels run ternary weights.
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"

namespace hq {

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvRowsPerCta = kGemvThreads / 32;

// Digits 0..4 of byte v in base 3, 2 bits each (the same digit arithmetic as
// native_decoder.cu:183-186 for every byte value, including v >= 243).
__device__ __forceinline__ uint32_t base3_digits(uint32_t v) {
    uint32_t d = 0;
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        d |= (v % 3u) << (2 * s);
        v /= 3u;
    }
    return d;
}

__device__ __forceinline__ float trit_times(uint32_t code, float x) {
    // code 0 -> -x, 1 -> 0, 2 -> +x
    return code == 2u ? x : (code == 0u ? -x : 0.0f);
}

__global__ void __launch_bounds__(kGemvThreads) tq1_0_gemv_kernel(const float* __restrict__ x,
                                                                  const uint8_t* __restrict__ w,
                                                                  float* __restrict__ out, int in_dim,
                                                                  int out_dim) {
    extern __shared__ float sx[];
    __shared__ uint16_t lut[256];
    for (int i = threadIdx.x; i < in_dim; i += blockDim.x) sx[i] = x[i];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = (uint16_t)base3_digits((uint32_t)i);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = in_dim / 256;
    const int blk_in_pass = lane / 7, part = lane % 7;  // lanes 0..27 active
    for (int row = blockIdx.x * kGemvRowsPerCta + warp; row < out_dim; row += gridDim.x * kGemvRowsPerCta) {
        const uint8_t* rowp = w + (size_t)row * nb * 56;
        float sum = 0.f;
        for (int b0 = 0; b0 < nb; b0 += 4) {
            const int b = b0 + blk_in_pass;
            float part_sum = 0.f;
            float d = 0.f;
            bool active = lane < 28 && b < nb;
            uint2 v = make_uint2(0, 0);
            if (active) v = __ldg(reinterpret_cast<const uint2*>(rowp + (size_t)b * 56 + part * 8));
            // d lives in bytes 0-1 of the block = low half of lane part 0's first word
            const int src_lane = blk_in_pass * 7;
            const uint32_t dbits = __shfl_sync(0xffffffffu, v.x, src_lane < 32 ? src_lane : 0);
            if (active) {
                d = __half2float(__ushort_as_half((unsigned short)(dbits & 0xFFFFu)));
                const float* xp = sx + b * 256;
                uint8_t bytes[8];
                *reinterpret_cast<uint2*>(bytes) = v;
                // block byte offset of bytes[0] is 8*part; packed index = offset - 2
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int pi = 8 * part + i - 2;  // packed index
                    if (pi < 0 || pi > 51) continue;
                    const uint32_t dig = lut[bytes[i]];
                    if (pi < 50) {
#pragma unroll
                        for (int s = 0; s < 5; ++s) part_sum += trit_times((dig >> (2 * s)) & 3u, xp[pi * 5 + s]);
                    } else {
#pragma unroll
                        for (int s = 0; s < 3; ++s)
                            part_sum += trit_times((dig >> (2 * s)) & 3u, xp[250 + (pi - 50) * 3 + s]);
                    }
                }
                if (isnan(d) || isinf(d)) part_sum = 0.f, d = 0.f;  // native_decoder.cu:174
            }
            sum = fmaf(d, part_sum, sum);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, off);
        if (lane == 0) out[row] = sum;
    }
}

// ---------------------------------------------------------------------------
// Tensor-core TQ1_0 GEMV.
//
// Row data is consumed in 32-byte windows: lane (g, t) of a warp owns bytes
// [8t, 8t+8) of each window of rows g and g + 8 of a 16-row unit.  A block
// (56 B) starts on an 8-byte boundary, so a lane's 8 bytes lie in one block,
// and a 32-byte window touches at most two consecutive blocks (one of each
// parity).  Four blocks (224 B, a "group") are seven windows: blocks 0..3
// start in windows 0, 1, 3, 5 (lanes 0, 3, 2, 1) and end in windows 1, 3, 5, 6.
//
// Operand A (16 rows x 32 k, u8) per lane and window: for each byte beta of the
// lane's 8, the register [d0, d1, d2, d3] of its digits, then [d4] of bytes 0-3
// and of bytes 4-7: ten registers, five mmas (registers 2m, 2m+1 of rows g and
// g + 8).  Operand B (32 k x 8 columns, s8): column 4P + p holds piece p of x
// at the position of each A slot whose byte lies in a block of parity P, zero
// elsewhere (and zero at the fp16 d bytes, the pad bytes and digits 3-4 of
// packed bytes 50-51).  B depends only on the window and the lane: it is built
// into shared memory for up to kChunkGroups groups of in_dim at a time
// (1280 B per window).
//
// Weights reach shared memory through the bulk-copy (TMA) engine: each warp
// has a private two-stage ring of (16 rows x 224 B) stages, one 224-byte copy
// per row, completion on a per-stage mbarrier.  The bytes in flight cost no
// registers, and the warp's first two stages are requested before the tables
// are built.  One CTA per SM: 16 warps share the tables.
// ---------------------------------------------------------------------------
constexpr int kTcWarps = 16;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kGroupBytes = 224;                  // 4 blocks of one row
constexpr int kStageBytes = 16 * kGroupBytes;     // one group of a 16-row unit
constexpr int kChunkGroups = 5;                   // groups per operand-B table (1280 in_dim)
constexpr int kBEntryBytes = 5 * 32 * 8;          // one window: 5 mmas x 32 lanes x (b0, b1)
constexpr int kLutBytes = 256 * 256;              // value v at [v * 256, v * 256 + 128): lane l's copy at + 4l
constexpr int kSmemB = kLutBytes;
constexpr int kSmemQ = kSmemB + kChunkGroups * 7 * kBEntryBytes;
constexpr int kSmemRing = kSmemQ + kChunkGroups * 4 * 16;
constexpr int kSmemBar = kSmemRing + kTcWarps * 2 * kStageBytes;
constexpr int kTcSmemBytes = kSmemBar + kTcWarps * 2 * 8;
static_assert(kSmemRing % 16 == 0 && kSmemBar % 8 == 0, "bulk-copy destinations and mbarriers alignment");

// Table word for byte value v: digits (v / 3^s) % 3 (the reference's digit
// arithmetic, native_decoder.cu:183-186, for every byte value) as
// d0 | d4 << 2 | d1 << 8 | d2 << 16 | d3 << 24.
__device__ __forceinline__ uint32_t tq1_digit_word(uint32_t v) {
    const uint32_t d0 = v % 3u, d1 = (v / 3u) % 3u, d2 = (v / 9u) % 3u, d3 = (v / 27u) % 3u, d4 = (v / 81u) % 3u;
    return d0 | (d4 << 2) | (d1 << 8) | (d2 << 16) | (d3 << 24);
}

// Offset within its block of the weight that A slot i of register r of a lane
// whose 8 bytes start at block byte ob feeds, or -1 for a slot that carries no
// weight (d bytes, pad bytes, digits 3-4 of packed bytes 50-51).
__device__ __forceinline__ int tq1_slot_k(int ob, int r, int i) {
    const int beta = r < 8 ? r : 4 * (r - 8) + i;
    const int s = r < 8 ? i : 4;
    const int p = ob + beta - 2;  // packed index
    if (p >= 0 && p < 50) return 5 * p + s;
    if ((p == 50 || p == 51) && s < 3) return 250 + 3 * (p - 50) + s;
    return -1;
}

// x * 2^sh rounded to an integer X (|X| <= 2^27), as balanced base-128 digits
// q0..q3 (X = ((q0 * 128 + q1) * 128 + q2) * 128 + q3, each in [-64, 64]) in bytes 0..3.
__device__ __forceinline__ uint32_t x_pieces(float v, int sh) {
    const int X = __float2int_rn(ldexpf(v, sh));
    const int q3 = ((X + 64) & 127) - 64;
    const int X1 = (X - q3) >> 7;
    const int q2 = ((X1 + 64) & 127) - 64;
    const int X2 = (X1 - q2) >> 7;
    const int q1 = ((X2 + 64) & 127) - 64;
    const int q0 = (X2 - q1) >> 7;
    return (uint32_t)(q0 & 0xFF) | ((uint32_t)(q1 & 0xFF) << 8) | ((uint32_t)(q2 & 0xFF) << 16) |
           ((uint32_t)(q3 & 0xFF) << 24);
}

__device__ __forceinline__ void imma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The reference's per-row loop (native_decoder.cu:171-199) for one row, x read
// from global memory: the path for an x that holds NaN or Inf.
__device__ float tq1_row_direct(const float* __restrict__ x, const uint8_t* __restrict__ rowp, int nb, int lane) {
    float sum = 0.f;
    for (int b = lane; b < nb; b += 32) {
        const uint8_t* blk = rowp + (size_t)b * 56;
        const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
        if (isnan(d) || isinf(d)) continue;
        const float* xp = x + (size_t)b * 256;
        for (int p = 0; p < 52; ++p) {
            uint32_t v = blk[2 + p];
            const int n = p < 50 ? 5 : 3;
            for (int s = 0; s < n; ++s) {
                const float trit = (float)((int)(v % 3u) - 1);
                v /= 3u;
                sum += (d * trit) * xp[p < 50 ? 5 * p + s : 250 + 3 * (p - 50) + s];
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, off);
    return sum;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tq1_0_gemv_tc_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w, float* __restrict__ out,
                         int in_dim, int out_dim, unsigned* __restrict__ err) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint32_t s_max[kTcWarps];
    __shared__ int s_bad[kTcWarps];
    __shared__ float s_part[kTcWarps][2][16];  // partial-unit row sums of a chunk (head, tail of each run)
    __shared__ int s_part_unit[kTcWarps][2];
    const uint8_t* lut = smem;                                    // digit table
    uint2* btab = reinterpret_cast<uint2*>(smem + kSmemB);       // [window of chunk][mma][lane]
    float4* qtab = reinterpret_cast<float4*>(smem + kSmemQ);     // [block of chunk] (Q0*128+Q1, Q2*128+Q3, -, -)
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
    const int nb = in_dim / 256, n_groups = nb / 4;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t row_bytes = (size_t)nb * 56;

    // 1. max|x| and finiteness
    uint32_t m = 0;
    int bad = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
        for (int i = tid; i < in_dim / 4; i += kTcThreads) {
            const float4 v = __ldg(x4 + i);
            bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
            m = max(m, max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                           max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w)))));
        }
    } else {  // x only 4-byte aligned
#pragma unroll 4
        for (int i = tid; i < in_dim; i += kTcThreads) {
            const float v = __ldg(x + i);
            bad |= !isfinite(v);
            m = max(m, __float_as_uint(fabsf(v)));
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        s_max[warp] = m;
        s_bad[warp] = bad;
        mbar_init(&bars[2 * warp], 1);
        mbar_init(&bars[2 * warp + 1], 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    m = 0;
    bad = 0;
#pragma unroll
    for (int i = 0; i < kTcWarps; ++i) m = max(m, s_max[i]), bad |= s_bad[i];
    if (bad) {  // NaN/Inf in x: the reference's float arithmetic, row by row
        for (int row = blockIdx.x * kTcWarps + warp; row < out_dim; row += gridDim.x * kTcWarps) {
            const float v = tq1_row_direct(x, w + (size_t)row * row_bytes, nb, lane);
            if (lane == 0) out[row] = v;
        }
        return;
    }
    int e = 0;
    frexpf(__uint_as_float(m), &e);  // max|x| < 2^e (e = 0 when x == 0)
    const int sh = 27 - e;

    // 2. work: the CTA's 16-row units [u_begin, u_begin + u_count).  Per chunk of kChunkGroups groups,
    //    the tasks (unit, group) in unit-major order are cut into kTcWarps contiguous runs, one per warp.
    //    The ring runs two tasks ahead of the decode, across chunk boundaries.
    const int n_units = (out_dim + 15) / 16;
    const int per_cta = (n_units + gridDim.x - 1) / gridDim.x;
    const int u_begin = blockIdx.x * per_cta;
    const int u_count = max(0, min(per_cta, n_units - u_begin));
    const int n_chunks = (n_groups + kChunkGroups - 1) / kChunkGroups;
    auto chunk_groups = [&](int c) { return min(kChunkGroups, n_groups - c * kChunkGroups); };
    auto run_of = [&](int c, int& t0, int& t1) {  // this warp's tasks of chunk c: [t0, t1)
        const int total = u_count * chunk_groups(c);
        const int T = (total + kTcWarps - 1) / kTcWarps;
        t0 = min(warp * T, total);
        t1 = min(t0 + T, total);
    };
    int n_steps = 0;
    for (int c = 0; c < n_chunks; ++c) {
        int a, b;
        run_of(c, a, b);
        n_steps += b - a;
    }
    uint8_t* ring = smem + kSmemRing + warp * 2 * kStageBytes;
    bool ok = true;
    int i_chunk = 0, i_task = 0, i_end = 0, i_unit = 0, i_grp = 0;  // issue cursor: next task to request
    run_of(0, i_task, i_end);
    i_unit = i_task / chunk_groups(0);
    i_grp = i_task - i_unit * chunk_groups(0);
    auto issue = [&](int st) {  // request the next task into stage st & 1 (st < n_steps)
        while (i_task == i_end && i_chunk + 1 < n_chunks) {
            ++i_chunk;
            run_of(i_chunk, i_task, i_end);
            i_unit = i_task / chunk_groups(i_chunk);
            i_grp = i_task - i_unit * chunk_groups(i_chunk);
        }
        const int unit = u_begin + i_unit;
        const int G = i_chunk * kChunkGroups + i_grp;
        ++i_task;
        if (++i_grp == chunk_groups(i_chunk)) i_grp = 0, ++i_unit;
        const int rows = min(16, out_dim - unit * 16);
        uint64_t* bar = &bars[2 * warp + (st & 1)];
        if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(rows * kGroupBytes));
        __syncwarp();
        if (lane < rows)
            bulk_g2s(ring + (st & 1) * kStageBytes + lane * kGroupBytes,
                     w + (size_t)(unit * 16 + lane) * row_bytes + (size_t)G * kGroupBytes, kGroupBytes, bar);
    };
    if (n_steps > 0) issue(0);
    if (n_steps > 1) issue(1);

    // 3. chunk 0's x pieces, converted once and coalesced, into the digit-table region (free until the
    //    table is built, after chunk 0's tables): its operand-B table and block sums then read shared memory.
    uint32_t* xq0 = reinterpret_cast<uint32_t*>(smem);
    const int k_chunk0 = min(in_dim, kChunkGroups * 4 * 256);
    for (int k = tid; k < k_chunk0; k += kTcThreads) xq0[k] = x_pieces(__ldg(x + k), sh);

    const int g = lane >> 2, t = lane & 3;
    const uint32_t lane_off = (uint32_t)lane * 4u;
    // this lane's C columns are pieces (p, p + 1) = 2 (t & 1) + (0, 1) of parity t >> 1; a block's
    // value for them is (C_p * 128 + C_{p+1}) - (Q_p * 128 + Q_{p+1}), weighted 2^14 (p = 0) or 1 (p = 2)
    const int lane_scale_exp = (t & 1) ? 0 : 14;
    const bool flush_even = (t >> 1) == 0;
    const uint32_t lut_s = smem_u32(lut);
    int st = 0;                                      // next step to decode
    for (int c = 0; c * kChunkGroups < n_groups; ++c) {
        const int n_cg = min(kChunkGroups, n_groups - c * kChunkGroups);
        __syncthreads();  // the previous chunk's tables are no longer read
        // 4. operand-B table and per-block piece sums of this chunk (chunk 0 from xq0, later ones from x)
        auto piece = [&](int k) { return c == 0 ? xq0[k] : x_pieces(__ldg(x + k), sh); };
        for (int idx = tid; idx < n_cg * 7 * 20; idx += kTcThreads) {
            const int j = idx / 20, mm = (idx / 4) % 5, tt = idx % 4;
            const int o = 32 * j + 8 * tt;  // chunk byte offset of lane tt's 8 bytes
            const int Gl = o / kGroupBytes, og = o % kGroupBytes, cb = og / 56, ob = og % 56;
            const int kbase = ((c * kChunkGroups + Gl) * 4 + cb) * 256, P = cb & 1;
            uint32_t v[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int kk = tq1_slot_k(ob, 2 * mm + h, i);
                    v[h][i] = kk < 0 ? 0u : piece(kbase + kk);
                }
            uint2* dst = btab + (size_t)(j * 5 + mm) * 32 + tt;
#pragma unroll
            for (int gg = 0; gg < 8; ++gg) {
                uint2 ent = make_uint2(0u, 0u);
                if ((gg >> 2) == P) {
                    const uint32_t sel = (uint32_t)(gg & 3) | ((uint32_t)(4 + (gg & 3)) << 4);
                    ent.x = __byte_perm(__byte_perm(v[0][0], v[0][1], sel), __byte_perm(v[0][2], v[0][3], sel), 0x5410);
                    ent.y = __byte_perm(__byte_perm(v[1][0], v[1][1], sel), __byte_perm(v[1][2], v[1][3], sel), 0x5410);
                }
                dst[gg * 4] = ent;
            }
        }
        for (int bl = warp; bl < n_cg * 4; bl += kTcWarps) {
            const int k0 = (c * kChunkGroups * 4 + bl) * 256 + lane * 8;
            int acc[4] = {0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t v = piece(k0 + i);
#pragma unroll
                for (int p = 0; p < 4; ++p) acc[p] += (int)(int8_t)(v >> (8 * p));
            }
#pragma unroll
            for (int p = 0; p < 4; ++p) acc[p] = __reduce_add_sync(0xffffffffu, acc[p]);
            // exact in fp32: |Q_p| <= 256 * 64, so |Q0 * 128 + Q1| < 2^22
            if (lane == 0) qtab[bl] = make_float4((float)(acc[0] * 128 + acc[1]), (float)(acc[2] * 128 + acc[3]), 0.f, 0.f);
        }
        __syncthreads();
        if (c == 0) {  // digit table: 16 byte values per warp, each stored to all 32 lane copies (over xq0)
            const uint32_t mine = tq1_digit_word((uint32_t)(warp * 16 + (lane & 15)));
#pragma unroll
            for (int i = 0; i < 16; ++i)
                reinterpret_cast<uint32_t*>(smem)[(warp * 16 + i) * 64 + lane] = __shfl_sync(0xffffffffu, mine, i);
            __syncthreads();
        }

        // 5. decode this warp's run of the chunk's tasks.  Row sums stay in registers while the unit
        //    is the same; a segment that covers the unit's whole chunk is added to out directly, a
        //    partial one (only at the run's head or tail) goes to s_part and is combined below.
        int t0, t1;
        run_of(c, t0, t1);
        if (lane == 0) s_part_unit[warp][0] = s_part_unit[warp][1] = -1;
        float y[2] = {0.f, 0.f};
        int seg_unit = -1, seg_start = t0;
        auto emit = [&](int seg_end) {  // tasks [seg_start, seg_end) of unit seg_unit
            const bool full = seg_start == seg_unit * n_cg && seg_end == seg_unit * n_cg + n_cg;
            const int slot = seg_start == t0 ? 0 : 1;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                float v = ldexpf(y[q], lane_scale_exp);
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v = ldexpf(v, e - 27);
                const int row = (u_begin + seg_unit) * 16 + g + 8 * q;
                if (t == 0) {
                    if (!full)
                        s_part[warp][slot][g + 8 * q] = v;
                    else if (row < out_dim)
                        out[row] = c == 0 ? v : out[row] + v;
                }
                y[q] = 0.f;
            }
            if (!full && lane == 0) s_part_unit[warp][slot] = seg_unit;
        };
        int ul = t0 / max(n_cg, 1), Gl = t0 - ul * n_cg;  // task = ul * n_cg + Gl
        for (int task = t0; task < t1; ++task, ++st, (++Gl == n_cg ? (Gl = 0, ++ul) : 0)) {
            if (ul != seg_unit) {
                if (seg_unit >= 0) emit(task);
                seg_unit = ul;
                seg_start = task;
            }
            float dsc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // block scale per parity and row
            int acc[4] = {0, 0, 0, 0};
            if (ok) ok = mbar_wait(&bars[2 * warp + (st & 1)], (uint32_t)((st >> 1) & 1), err);
            const uint32_t sp = smem_u32(ring + (st & 1) * kStageBytes + 8 * t);
#pragma unroll
            for (int win = 0; win < 7; ++win) {
                uint2 wv[2];
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(wv[q].x), "=r"(wv[q].y)
                        : "r"(sp + (g + 8 * q) * kGroupBytes + 32 * win));
                if (win == 0 || win == 1 || win == 3 || win == 5) {  // a block starts: take its d
                    const int blk = win == 0 ? 0 : win == 1 ? 1 : win == 3 ? 2 : 3;
                    const int src = (lane & ~3) | (win == 0 ? 0 : win == 1 ? 3 : win == 3 ? 2 : 1);
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const uint32_t bits = __shfl_sync(0xffffffffu, wv[q].x, src);
                        const float d = __half2float(__ushort_as_half((unsigned short)(bits & 0xFFFFu)));
                        dsc[blk & 1][q] = fabsf(d) <= 65504.f ? d : 0.f;  // NaN/Inf: skipped, native_decoder.cu:174
                    }
                }
                uint32_t R[2][10];  // A registers of rows g, g + 8
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    uint32_t T[8];
#pragma unroll
                    for (int beta = 0; beta < 8; ++beta) {
                        const uint32_t word = beta < 4 ? wv[q].x : wv[q].y;
                        const uint32_t off = __byte_perm(word, lane_off, 0x5504u | ((uint32_t)(beta & 3) << 4));
                        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(T[beta]) : "r"(lut_s + off));
                        R[q][beta] = T[beta] & 0x03030303u;
                    }
                    R[q][8] = (__byte_perm(__byte_perm(T[0], T[1], 0x0040), __byte_perm(T[2], T[3], 0x0040),
                                           0x5410) >> 2) & 0x03030303u;
                    R[q][9] = (__byte_perm(__byte_perm(T[4], T[5], 0x0040), __byte_perm(T[6], T[7], 0x0040),
                                           0x5410) >> 2) & 0x03030303u;
                }
                const uint32_t bw = smem_u32(btab) + (uint32_t)((((Gl * 7 + win) * 5) * 32 + lane) * 8);
#pragma unroll
                for (int mm = 0; mm < 5; ++mm) {
                    uint2 b;
                    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(b.x), "=r"(b.y) : "r"(bw + mm * 256));
                    imma_u8s8(acc, R[0][2 * mm], R[1][2 * mm], R[0][2 * mm + 1], R[1][2 * mm + 1], b.x, b.y);
                }
                if (win == 1 || win == 3 || win == 5 || win == 6) {  // a block ends: fold it in
                    const int blk = win == 1 ? 0 : win == 3 ? 1 : win == 5 ? 2 : 3;
                    if (flush_even == ((blk & 1) == 0)) {
                        const float2 qs = *reinterpret_cast<const float2*>(&qtab[4 * Gl + blk]);
                        const float qf = (t & 1) ? qs.y : qs.x;
#pragma unroll
                        for (int q = 0; q < 2; ++q) {  // |C_p * 128 + C_{p+1}| < 2^23: exact in fp32
                            const float v = (float)(acc[2 * q] * 128 + acc[2 * q + 1]) - qf;
                            y[q] = fmaf(dsc[blk & 1][q], v, y[q]);
                            acc[2 * q] = 0;
                            acc[2 * q + 1] = 0;
                        }
                    }
                }
            }
            __syncwarp();  // every lane is done with this stage
            if (ok && st + 2 < n_steps) issue(st + 2);
        }
        if (seg_unit >= 0) emit(t1);
        __syncthreads();
        if (warp == 0 && lane < 16) {  // partial segments, unit by unit in warp order (deterministic)
            int cur = -1;
            float sum = 0.f;
            auto put = [&]() {
                const int row = (u_begin + cur) * 16 + lane;
                if (row < out_dim) out[row] = c == 0 ? sum : out[row] + sum;
            };
            for (int ww = 0; ww < kTcWarps; ++ww)
#pragma unroll
                for (int sl = 0; sl < 2; ++sl) {
                    const int u = s_part_unit[ww][sl];
                    if (u < 0) continue;
                    if (u != cur) {
                        if (cur >= 0) put();
                        cur = u;
                        sum = 0.f;
                    }
                    sum += s_part[ww][sl][lane];
                }
            if (cur >= 0) put();
        }
    }
}

// One thread per tile word (s, kb, lane, j) + the scale array.
__global__ void tq1_0_to_tile_t2_kernel(const uint8_t* __restrict__ w, uint32_t* __restrict__ tile,
                                        uint16_t* __restrict__ scales, int K, int N) {
    const TileGeom geo(K, N, 2);
    const int nb = K / 256;
    const size_t total = geo.bytes() / 4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += stride) {
        const size_t chunk = i / 64;
        const int within = (int)(i % 64);
        const int lane = within / 2, j = within % 2;
        const size_t per_full_group = (size_t)kGroupStrips * geo.KB;
        const int sg = (int)(chunk / per_full_group);
        const size_t rem = chunk - (size_t)sg * per_full_group;
        const int wd = geo.width(sg);
        const int kb = (int)(rem / wd), sl = (int)(rem % wd);
        int col, kw;
        tile_word_source(2, sg * kGroupStrips + sl, kb, lane, j, &col, &kw);
        const int k0 = kw * 16;
        const uint8_t* blk = w + ((size_t)col * nb + k0 / 256) * 56;
        uint32_t lin = 0;
        for (int e = 0; e < 16; ++e) {
            const int el = (k0 % 256) + e;
            const int by = el < 250 ? el / 5 : 50 + (el - 250) / 3;
            const int dg = el < 250 ? el % 5 : (el - 250) % 3;
            uint32_t v = blk[2 + by];
            for (int s = 0; s < dg; ++s) v /= 3u;
            lin |= (v % 3u) << (2 * e);  // code = trit + 1
        }
        tile[i] = t2_linear_to_tile(lin);
    }
    const size_t ns = (size_t)(K / 128) * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < ns; i += stride) {
        const int gi = (int)(i / N), n = (int)(i % N);
        const uint8_t* blk = w + ((size_t)n * nb + gi / 2) * 56;
        uint16_t d = (uint16_t)(blk[0] | (blk[1] << 8));
        if ((d & 0x7C00u) == 0x7C00u) d = 0;  // NaN/Inf block: contributes nothing
        scales[i] = d;
    }
}

}  // namespace

cudaError_t launch_tq1_0_gemv(const float* x, const uint8_t* w, float* out, int in_dim, int out_dim,
                              cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const DeviceInfo& di = device_info(dev);
    if (in_dim % 1024 == 0 && (size_t)kTcSmemBytes + 4096 <= di.smem_optin && (reinterpret_cast<uintptr_t>(w) & 15u) == 0) {
        e = ensure_smem_attr(reinterpret_cast<const void*>(tq1_0_gemv_tc_kernel), dev, kTcSmemBytes);
        if (e != cudaSuccess) return e;
        const int units = (out_dim + 15) / 16;
        const int grid = units < di.sm_count ? units : di.sm_count;  // one CTA per SM
        tq1_0_gemv_tc_kernel<<<grid, kTcThreads, kTcSmemBytes, s>>>(x, w, out, in_dim, out_dim, device_error_word(dev));
        return cudaGetLastError();
    }
    const size_t smem = (size_t)in_dim * sizeof(float);
    e = ensure_smem_attr(reinterpret_cast<const void*>(tq1_0_gemv_kernel), dev, (int)smem);
    if (e != cudaSuccess) return e;
    const int blocks_needed = (out_dim + kGemvRowsPerCta - 1) / kGemvRowsPerCta;
    const int grid = blocks_needed < device_info(dev).sm_count * 8 ? blocks_needed : device_info(dev).sm_count * 8;
    tq1_0_gemv_kernel<<<grid, kGemvThreads, smem, s>>>(x, w, out, in_dim, out_dim);
    return cudaGetLastError();
}

cudaError_t launch_tq1_0_to_tile_t2(const uint8_t* w, uint8_t* tile, uint16_t* scales, int K, int N,
                                    cudaStream_t s) {
    const TileGeom geo(K, N, 2);
    size_t total = geo.bytes() / 4;
    int grid = (int)((total + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    tq1_0_to_tile_t2_kernel<<<grid, 256, 0, s>>>(w, reinterpret_cast<uint32_t*>(tile), scales, K, N);
    return cudaGetLastError();
}

}  // namespace hq
