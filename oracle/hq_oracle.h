/*
 * hq_oracle.h -- CPU restatement of the reference's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library (nebula_b200/,
 * libhq.so) links, loads or calls this code.  Only tests/, the smoke() check in
 * __graft_entry__.py and the cpu_baseline / --impl reference legs of bench.py
 * use it, and only as the checker or as the timed CPU baseline.
 *
 * Every routine names the reference source it restates (paths relative to the
 * Nebula project root).  Pinning: the int4 repack is checked bit-exactly against
 * the reference's own MarlinGemmEngine::repack_q4k_to_marlin compiled from
 * source (oracle/_ref), and the fp32 dequant-then-matmul is checked bit-exactly
 * against the reference's kernel_reference_gemm run on a B200 through the same
 * compiled library.  The TQ1_0 routines follow native_decoder.cu line by line;
 * that file cannot be compiled outside Windows, so TQ1_0 parity is pinned by the
 * restatement only.  The 2-bit "T2" and "tile" formats are defined by this
 * project (not present in the reference): unpinned by the reference.
 */
#ifndef HQ_ORACLE_H
#define HQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- formats */

/* Linear int4: uint32 [K/8][N]; word (kw,n) holds k = 8*kw + i at bits 4i,
 * code u = q + 8 in [0,15].  Follows marlin_gemm.cu:495-510. */
int hqo_pack_linear_u4(const int8_t* q, uint32_t* out, int K, int N);
int hqo_unpack_linear_u4(const uint32_t* w, int8_t* q, int K, int N);

/* Reference "Marlin quad" layout: uint4 [K/32][N]; quad (kq,n) word j is the
 * linear word (4*kq + j, n).  Follows marlin_gemm.cu:446-455. */
int hqo_repack_marlin_quad(const uint32_t* linear, uint32_t* quad, int K, int N);
int hqo_unrepack_marlin_quad(const uint32_t* quad, uint32_t* linear, int K, int N);

/* Linear 2-bit ternary ("T2"): uint32 [K/16][N]; word (kw,n) holds
 * k = 16*kw + i at bits 2i, code c = t + 1 in {0,1,2}. */
int hqo_pack_linear_t2(const int8_t* t, uint32_t* out, int K, int N);
int hqo_unpack_linear_t2(const uint32_t* w, int8_t* t, int K, int N);

/* Tile format used by the CUDA kernels (this project's layout; the exact
 * byte map is documented in hq_oracle.c above hqo_tile_word_index). wbits is 4
 * (int4, q in [-8,7]) or 2 (ternary, q in [-1,1]).  q is [K][N] row-major. */
size_t hqo_tile_bytes(int K, int N, int wbits);
int hqo_pack_tile(const int8_t* q, uint8_t* tile, int K, int N, int wbits);
int hqo_unpack_tile(const uint8_t* tile, int8_t* q, int K, int N, int wbits);

/* TQ1_0 (native_decoder.cu:32-36, element decode :81-101, :179-198):
 * [N rows][K/256 blocks] of 56 bytes {fp16 d; uint8 packed[52]; uint16 pad}.
 * t is [N][K] row-major (one row per output), d_bits is [N][K/256]. */
int hqo_pack_tq1_0(const int8_t* t, const uint16_t* d_bits, uint8_t* out, int K, int N);
int hqo_unpack_tq1_0(const uint8_t* in, int8_t* t, uint16_t* d_bits, int K, int N);

/* ------------------------------------------------------------------- math */

/* fp16 bits -> float (exact). */
float hqo_half_to_float(uint16_t h);

/* W[k][n] = (float)u * scale + bias (two roundings), the reference's host
 * dequant (marlin_gemm.cu:506); with bias == NULL the symmetric form
 * W = (float)(u - 8) * scale (one rounding) is used instead. */
int hqo_dequant_u4(const uint32_t* linear, const float* scales, const float* bias,
                   float* W, int K, int N, int group);

/* Y[m][n] = sum_k X[m][k] * W[k][n], fp32, k ascending, each step one fused
 * multiply-add: kernel_reference_gemm (marlin_gemm.cu:52-70) as nvcc compiles
 * it (the a*b+c in :66 contracts to an FMA). */
int hqo_gemm_f32(const float* X, const float* W, float* Y, int M, int K, int N,
                 int nthreads);

/* Fused dequant + matmul, bit-identical to hqo_dequant_u4 + hqo_gemm_f32. */
int hqo_w4_gemm(const float* X, const uint32_t* linear, const float* scales,
                const float* bias, float* Y, int M, int K, int N, int group,
                int nthreads);

/* Ternary linear T2 GEMM: W = (float)t * scale, fp32 FMA, k ascending. */
int hqo_t2_gemm(const float* X, const uint32_t* linear_t2, const float* scales,
                float* Y, int M, int K, int N, int group, int nthreads);

/* kernel_gemv_tq1_0 (native_decoder.cu:155-206) including its 32-lane
 * partial sums, its per-block NaN/Inf skip (:174) and the shuffle-down
 * reduction tree (:39-45).  Computes every row (the reference launch geometry
 * at :1090-1091 leaves rows uncomputed; that launch bug is not restated). */
int hqo_gemv_tq1_0(const float* x, const uint8_t* w, float* out, int in_dim,
                   int out_dim, int nthreads);

/* kernel_cutlass_int8_gemm (marlin_gemm.cu:327-377), one output at a time:
 * q8(x) = (int8) trunc(clamp(x * 127, -128, 127)) per element; per quad of k
 * the 4-lane int8 dot product, added to an fp32 running sum as
 * fmaf((float)dot, 1/127, acc) (nvcc's contraction of :369); the K % 4 tail is
 * ignored as in the reference; Y = acc * scale[n].  W int8 [K][N]. */
int hqo_w8_gemm(const float* X, const int8_t* W, const float* scales, float* Y,
                int M, int K, int N, int nthreads);

/* GGML tensor types taken by the projection routines (gguf_parser.hpp:33-64). */
#define HQO_GGML_F32 0
#define HQO_GGML_Q8_0 8
#define HQO_GGML_BF16 30
#define HQO_GGML_TQ1_0 34
#define HQO_GGML_TQ1_0_ALT 143 /* also read as TQ1_0 (forward_baseline.cu:82,218) */

/* kernel_output_projection (forward_baseline.cu:178-257): logits[row] =
 * dot(W[row, :], x), one warp per row.  Restated with its 32 lane partial sums
 * (F32 / BF16: elements lane + 32 i; Q8_0: blocks lane + 32 i, element order
 * within a block; TQ1_0: every block, packed bytes lane and lane + 32 below 50,
 * lanes 0-1 bytes 50-51), its fp32 arithmetic with the multiply-adds fused the
 * way nvcc contracts them, and the shuffle-down tree (:42-48).  Q8_0 applies d
 * unchecked; TQ1_0 replaces a NaN/Inf d by 0 (:223).  W rows: F32 / BF16
 * embedding_dim elements, Q8_0 embedding_dim/32 blocks of 34 bytes, TQ1_0
 * embedding_dim/256 blocks of 56 bytes. */
int hqo_output_projection(const float* x, const void* w, int type, float* logits,
                          int embedding_dim, int vocab_size, int nthreads);

/* kernel_embedding_lookup (forward_baseline.cu:55-109): row token_id of the
 * table, dequantised to fp32 (Q8_0: d * q; TQ1_0: d * trit with a NaN/Inf d
 * replaced by 0, as native_decoder.cu:63-103). */
int hqo_embedding_lookup(const void* table, int type, int token_id, float* out,
                         int embedding_dim);

#ifdef __cplusplus
}
#endif
#endif
