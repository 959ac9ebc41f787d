/*
 * hq_oracle.c -- CPU restatement of the reference's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY (see hq_oracle.h).  The product library never
 * links or loads this file; tests, smoke() and bench.py's CPU-baseline legs
 * use it as the checker / timed CPU baseline.
 *
 * Build: gcc -O3 -march=x86-64-v3 -ffp-contract=off -fopenmp -shared -fPIC
 * (oracle/build.py).  x86-64-v3 gives hardware FMA so fmaf() is one fused
 * operation, which lets hqo_gemm_f32 reproduce kernel_reference_gemm bit for
 * bit; -ffp-contract=off keeps every other a*b+c as two roundings, as the
 * reference's host dequant (marlin_gemm.cu:506) computes it.
 */
#include "hq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define HQO_EINVAL (-1)

static int set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    return nthreads;
#else
    (void)nthreads;
    return 1;
#endif
}

/* ------------------------------------------------------------ fp16 helper */

float hqo_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; ++e; } while ((man & 0x400) == 0);
            man &= 0x3FF;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* --------------------------------------------------------- linear formats */

/* marlin_gemm.cu:495-510: packed |= q << (i*4) for k = kw*8 + i, column n. */
int hqo_pack_linear_u4(const int8_t* q, uint32_t* out, int K, int N) {
    if (K <= 0 || N <= 0 || K % 8) return HQO_EINVAL;
    for (int kw = 0; kw < K / 8; ++kw)
        for (int n = 0; n < N; ++n) {
            uint32_t packed = 0;
            for (int i = 0; i < 8; ++i) {
                int v = q[(size_t)(kw * 8 + i) * N + n];
                if (v < -8 || v > 7) return HQO_EINVAL;
                packed |= (uint32_t)(v + 8) << (i * 4);
            }
            out[(size_t)kw * N + n] = packed;
        }
    return 0;
}

int hqo_unpack_linear_u4(const uint32_t* w, int8_t* q, int K, int N) {
    if (K <= 0 || N <= 0 || K % 8) return HQO_EINVAL;
    for (int kw = 0; kw < K / 8; ++kw)
        for (int n = 0; n < N; ++n) {
            uint32_t packed = w[(size_t)kw * N + n];
            for (int i = 0; i < 8; ++i)
                q[(size_t)(kw * 8 + i) * N + n] = (int8_t)(((packed >> (4 * i)) & 0xF) - 8);
        }
    return 0;
}

/* marlin_gemm.cu:446-455: dst[(kq*N + n)*4 + j] = src[(kq*4 + j)*N + n]. */
int hqo_repack_marlin_quad(const uint32_t* linear, uint32_t* quad, int K, int N) {
    if (K <= 0 || N <= 0 || K % 32) return HQO_EINVAL;
    for (int kq = 0; kq < K / 32; ++kq)
        for (int n = 0; n < N; ++n)
            for (int j = 0; j < 4; ++j)
                quad[((size_t)kq * N + n) * 4 + j] = linear[((size_t)kq * 4 + j) * N + n];
    return 0;
}

int hqo_unrepack_marlin_quad(const uint32_t* quad, uint32_t* linear, int K, int N) {
    if (K <= 0 || N <= 0 || K % 32) return HQO_EINVAL;
    for (int kq = 0; kq < K / 32; ++kq)
        for (int n = 0; n < N; ++n)
            for (int j = 0; j < 4; ++j)
                linear[((size_t)kq * 4 + j) * N + n] = quad[((size_t)kq * N + n) * 4 + j];
    return 0;
}

int hqo_pack_linear_t2(const int8_t* t, uint32_t* out, int K, int N) {
    if (K <= 0 || N <= 0 || K % 16) return HQO_EINVAL;
    for (int kw = 0; kw < K / 16; ++kw)
        for (int n = 0; n < N; ++n) {
            uint32_t packed = 0;
            for (int i = 0; i < 16; ++i) {
                int v = t[(size_t)(kw * 16 + i) * N + n];
                if (v < -1 || v > 1) return HQO_EINVAL;
                packed |= (uint32_t)(v + 1) << (i * 2);
            }
            out[(size_t)kw * N + n] = packed;
        }
    return 0;
}

int hqo_unpack_linear_t2(const uint32_t* w, int8_t* t, int K, int N) {
    if (K <= 0 || N <= 0 || K % 16) return HQO_EINVAL;
    for (int kw = 0; kw < K / 16; ++kw)
        for (int n = 0; n < N; ++n) {
            uint32_t packed = w[(size_t)kw * N + n];
            for (int i = 0; i < 16; ++i) {
                int c = (packed >> (2 * i)) & 3;
                if (c == 3) return HQO_EINVAL;
                t[(size_t)(kw * 16 + i) * N + n] = (int8_t)(c - 1);
            }
        }
    return 0;
}

/* ------------------------------------------------------------ tile format
 *
 * Strip s covers output columns [16s, 16s+16); strip group sg = s/8 holds
 * w_sg = min(8, N/16 - 8*sg) strips; k-block kb covers k in [64kb, 64kb+64).
 * A chunk (s, kb) is CB bytes (512 for int4, 256 for ternary) at byte offset
 *     (sg*8*KB + kb*w_sg + s%8) * CB,           KB = K/64,
 * so one strip group's chunks for consecutive kb are one contiguous run.
 * Inside a chunk, lane l = 4g + t (g in 0..7, t in 0..3) owns CB/32 bytes at
 * offset l*CB/32, laid out as 32-bit little-endian words:
 *   int4 (4 words): word j holds row r = g + 8*(j>>1), k offsets
 *       16t + 8*(j&1) + e for e = 0..7, the 4-bit code u = q + 8 of offset e
 *       at nibble position 2*((e>>1)&1) + ((e>>2)&1) + 4*(e&1)
 *       (e = 0..7 -> nibbles 0 4 2 6 1 5 3 7);
 *   ternary (2 words): word j holds row r = g + 8*j, k offsets 16t + e for
 *       e = 0..15, the 2-bit code c = q + 1 of offset e at field position
 *       (e>>1) + 8*(e&1).
 * "row r" is output column 16s + r.  The field order puts the codes of k and
 * k+1 sixteen bits apart, which is what a single masked OR with a floating
 * point exponent pattern turns into a half2/bf162 pair; in int4 words the
 * pairs (0,1),(2,3) use the low nibble of each byte and (4,5),(6,7) the high
 * nibble.
 */
size_t hqo_tile_bytes(int K, int N, int wbits) {
    if (K <= 0 || N <= 0 || K % 64 || N % 16 || (wbits != 4 && wbits != 2)) return 0;
    return (size_t)(K / 64) * (size_t)(N / 16) * (size_t)(wbits == 4 ? 512 : 256);
}

/* Byte offset of the 32-bit word holding (k, n) and the bit shift of its field. */
static size_t tile_locate(int k, int n, int K, int N, int wbits, int* shift) {
    const int KB = K / 64, NS = N / 16;
    const int s = n / 16, r = n % 16, kb = k / 64, ko = k % 64;
    const int sg = s / 8;
    const int wsg = (NS - 8 * sg) < 8 ? (NS - 8 * sg) : 8;
    const size_t CB = wbits == 4 ? 512 : 256;
    const size_t chunk = ((size_t)sg * 8 * KB + (size_t)kb * wsg + (size_t)(s % 8)) * CB;
    const int g = r % 8, t = ko / 16;
    const int lane = 4 * g + t;
    const size_t lane_off = chunk + (size_t)lane * (CB / 32);
    if (wbits == 4) {
        const int half = (ko % 16) / 8, e = ko % 8;
        const int j = 2 * (r / 8) + half;
        *shift = 4 * (2 * ((e >> 1) & 1) + ((e >> 2) & 1) + 4 * (e & 1));
        return lane_off + 4 * (size_t)j;
    } else {
        const int e = ko % 16;
        const int j = r / 8;
        *shift = 2 * ((e >> 1) + 8 * (e & 1));
        return lane_off + 4 * (size_t)j;
    }
}

int hqo_pack_tile(const int8_t* q, uint8_t* tile, int K, int N, int wbits) {
    size_t bytes = hqo_tile_bytes(K, N, wbits);
    if (!bytes) return HQO_EINVAL;
    memset(tile, 0, bytes);
    const int lo = wbits == 4 ? -8 : -1, hi = wbits == 4 ? 7 : 1, bias = -lo;
    for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n) {
            int v = q[(size_t)k * N + n];
            if (v < lo || v > hi) return HQO_EINVAL;
            int sh;
            size_t off = tile_locate(k, n, K, N, wbits, &sh);
            uint32_t word;
            memcpy(&word, tile + off, 4);
            word |= (uint32_t)(v + bias) << sh;
            memcpy(tile + off, &word, 4);
        }
    return 0;
}

int hqo_unpack_tile(const uint8_t* tile, int8_t* q, int K, int N, int wbits) {
    if (!hqo_tile_bytes(K, N, wbits)) return HQO_EINVAL;
    const uint32_t mask = wbits == 4 ? 0xF : 0x3;
    const int bias = wbits == 4 ? 8 : 1;
    for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n) {
            int sh;
            size_t off = tile_locate(k, n, K, N, wbits, &sh);
            uint32_t word;
            memcpy(&word, tile + off, 4);
            int c = (int)((word >> sh) & mask);
            if (wbits == 2 && c == 3) return HQO_EINVAL;
            q[(size_t)k * N + n] = (int8_t)(c - bias);
        }
    return 0;
}

/* ------------------------------------------------------------------ TQ1_0 */

/* Element j of a block: bytes 0..49 hold 5 trits (j/5, trit j%5), bytes 50..51
 * hold 3 trits (50 + (j-250)/3, trit (j-250)%3); least significant trit first,
 * trit value = digit - 1.  native_decoder.cu:81-101 and :179-198. */
static void tq1_pos(int j, int* byte, int* digit) {
    if (j < 250) { *byte = j / 5; *digit = j % 5; }
    else { *byte = 50 + (j - 250) / 3; *digit = (j - 250) % 3; }
}

int hqo_pack_tq1_0(const int8_t* t, const uint16_t* d_bits, uint8_t* out, int K, int N) {
    if (K <= 0 || N <= 0 || K % 256) return HQO_EINVAL;
    const int nb = K / 256;
    static const int pow3[5] = {1, 3, 9, 27, 81};
    for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b) {
            uint8_t* blk = out + ((size_t)n * nb + b) * 56;
            memset(blk, 0, 56);
            uint16_t d = d_bits[(size_t)n * nb + b];
            blk[0] = (uint8_t)(d & 0xFF);
            blk[1] = (uint8_t)(d >> 8);
            int acc[52] = {0};
            for (int j = 0; j < 256; ++j) {
                int v = t[(size_t)n * K + b * 256 + j];
                if (v < -1 || v > 1) return HQO_EINVAL;
                int by, dg;
                tq1_pos(j, &by, &dg);
                acc[by] += (v + 1) * pow3[dg];
            }
            for (int i = 0; i < 52; ++i) blk[2 + i] = (uint8_t)acc[i];
        }
    return 0;
}

int hqo_unpack_tq1_0(const uint8_t* in, int8_t* t, uint16_t* d_bits, int K, int N) {
    if (K <= 0 || N <= 0 || K % 256) return HQO_EINVAL;
    const int nb = K / 256;
    for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = in + ((size_t)n * nb + b) * 56;
            d_bits[(size_t)n * nb + b] = (uint16_t)(blk[0] | (blk[1] << 8));
            for (int j = 0; j < 256; ++j) {
                int by, dg;
                tq1_pos(j, &by, &dg);
                uint32_t val = blk[2 + by];
                for (int s = 0; s < dg; ++s) val /= 3;
                t[(size_t)n * K + b * 256 + j] = (int8_t)((int)(val % 3) - 1);
            }
        }
    return 0;
}

/* ------------------------------------------------------------------- math */

int hqo_dequant_u4(const uint32_t* linear, const float* scales, const float* bias,
                   float* W, int K, int N, int group) {
    if (K <= 0 || N <= 0 || K % 8 || group <= 0 || K % group || group % 8) return HQO_EINVAL;
    for (int kw = 0; kw < K / 8; ++kw)
        for (int n = 0; n < N; ++n) {
            uint32_t packed = linear[(size_t)kw * N + n];
            int gi = (kw * 8) / group;
            float s = scales[(size_t)gi * N + n];
            for (int i = 0; i < 8; ++i) {
                uint32_t u = (packed >> (4 * i)) & 0xF;
                float w;
                if (bias) {
                    const float prod = (float)u * s; /* rounded: built with -ffp-contract=off */
                    w = prod + bias[(size_t)gi * N + n];
                } else {
                    w = (float)((int)u - 8) * s;
                }
                W[(size_t)(kw * 8 + i) * N + n] = w;
            }
        }
    return 0;
}

/* Column-blocked so each output's k loop stays in ascending order while the
 * inner n loop vectorises; one fmaf per step as in marlin_gemm.cu:66. */
#define HQO_NB 256

int hqo_gemm_f32(const float* X, const float* W, float* Y, int M, int K, int N,
                 int nthreads) {
    if (M <= 0 || K <= 0 || N <= 0) return HQO_EINVAL;
    nthreads = set_threads(nthreads);
    const int nblocks = (N + HQO_NB - 1) / HQO_NB;
    #pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1) collapse(2)
    for (int m = 0; m < M; ++m)
        for (int nb = 0; nb < nblocks; ++nb) {
            const int n0 = nb * HQO_NB;
            const int n1 = n0 + HQO_NB < N ? n0 + HQO_NB : N;
            float acc[HQO_NB];
            for (int n = n0; n < n1; ++n) acc[n - n0] = 0.0f;
            for (int k = 0; k < K; ++k) {
                const float x = X[(size_t)m * K + k];
                const float* wr = W + (size_t)k * N;
                for (int n = n0; n < n1; ++n) acc[n - n0] = fmaf(x, wr[n], acc[n - n0]);
            }
            for (int n = n0; n < n1; ++n) Y[(size_t)m * N + n] = acc[n - n0];
        }
    return 0;
}

#define HQO_MB 16

int hqo_w4_gemm(const float* X, const uint32_t* linear, const float* scales,
                const float* bias, float* Y, int M, int K, int N, int group,
                int nthreads) {
    if (M <= 0 || K <= 0 || N <= 0 || K % 8 || group <= 0 || K % group || group % 8)
        return HQO_EINVAL;
    nthreads = set_threads(nthreads);
    const int nblocks = (N + HQO_NB - 1) / HQO_NB;
    const int mblocks = (M + HQO_MB - 1) / HQO_MB;
    #pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1) collapse(2)
    for (int mb = 0; mb < mblocks; ++mb)
        for (int nb = 0; nb < nblocks; ++nb) {
            const int m0 = mb * HQO_MB, m1 = m0 + HQO_MB < M ? m0 + HQO_MB : M;
            const int n0 = nb * HQO_NB, n1 = n0 + HQO_NB < N ? n0 + HQO_NB : N;
            const int nn = n1 - n0;
            float acc[HQO_MB][HQO_NB];
            float wk[HQO_NB];
            for (int m = m0; m < m1; ++m)
                for (int n = 0; n < nn; ++n) acc[m - m0][n] = 0.0f;
            for (int kw = 0; kw < K / 8; ++kw) {
                const int gi = (kw * 8) / group;
                const uint32_t* wrow = linear + (size_t)kw * N + n0;
                const float* srow = scales + (size_t)gi * N + n0;
                const float* brow = bias ? bias + (size_t)gi * N + n0 : 0;
                for (int i = 0; i < 8; ++i) {
                    const int k = kw * 8 + i;
                    if (brow) {
                        for (int n = 0; n < nn; ++n) {
                            float prod = (float)((wrow[n] >> (4 * i)) & 0xF) * srow[n];
                            wk[n] = prod + brow[n];
                        }
                    } else {
                        for (int n = 0; n < nn; ++n)
                            wk[n] = (float)((int)((wrow[n] >> (4 * i)) & 0xF) - 8) * srow[n];
                    }
                    for (int m = m0; m < m1; ++m) {
                        const float x = X[(size_t)m * K + k];
                        float* a = acc[m - m0];
                        for (int n = 0; n < nn; ++n) a[n] = fmaf(x, wk[n], a[n]);
                    }
                }
            }
            for (int m = m0; m < m1; ++m)
                for (int n = 0; n < nn; ++n) Y[(size_t)m * N + n0 + n] = acc[m - m0][n];
        }
    return 0;
}

int hqo_t2_gemm(const float* X, const uint32_t* linear_t2, const float* scales,
                float* Y, int M, int K, int N, int group, int nthreads) {
    if (M <= 0 || K <= 0 || N <= 0 || K % 16 || group <= 0 || K % group || group % 16)
        return HQO_EINVAL;
    nthreads = set_threads(nthreads);
    const int nblocks = (N + HQO_NB - 1) / HQO_NB;
    const int mblocks = (M + HQO_MB - 1) / HQO_MB;
    #pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1) collapse(2)
    for (int mb = 0; mb < mblocks; ++mb)
        for (int nb = 0; nb < nblocks; ++nb) {
            const int m0 = mb * HQO_MB, m1 = m0 + HQO_MB < M ? m0 + HQO_MB : M;
            const int n0 = nb * HQO_NB, n1 = n0 + HQO_NB < N ? n0 + HQO_NB : N;
            const int nn = n1 - n0;
            float acc[HQO_MB][HQO_NB];
            float wk[HQO_NB];
            for (int m = m0; m < m1; ++m)
                for (int n = 0; n < nn; ++n) acc[m - m0][n] = 0.0f;
            for (int kw = 0; kw < K / 16; ++kw) {
                const int gi = (kw * 16) / group;
                const uint32_t* wrow = linear_t2 + (size_t)kw * N + n0;
                const float* srow = scales + (size_t)gi * N + n0;
                for (int i = 0; i < 16; ++i) {
                    const int k = kw * 16 + i;
                    for (int n = 0; n < nn; ++n)
                        wk[n] = (float)((int)((wrow[n] >> (2 * i)) & 3) - 1) * srow[n];
                    for (int m = m0; m < m1; ++m) {
                        const float x = X[(size_t)m * K + k];
                        float* a = acc[m - m0];
                        for (int n = 0; n < nn; ++n) a[n] = fmaf(x, wk[n], a[n]);
                    }
                }
            }
            for (int m = m0; m < m1; ++m)
                for (int n = 0; n < nn; ++n) Y[(size_t)m * N + n0 + n] = acc[m - m0][n];
        }
    return 0;
}

/* native_decoder.cu:155-206.  Lane `lane` accumulates blocks lane, lane+32, ...
 * with sum = fma(d*trit, x, sum) per element in byte order; blocks whose d is
 * NaN or Inf are skipped (:174); the 32 partials are combined by the
 * shuffle-down tree of warp_reduce_sum (:39-45), whose lane-0 result is the
 * output. */
int hqo_gemv_tq1_0(const float* x, const uint8_t* w, float* out, int in_dim,
                   int out_dim, int nthreads) {
    if (in_dim <= 0 || out_dim <= 0 || in_dim % 256) return HQO_EINVAL;
    nthreads = set_threads(nthreads);
    const int nb = in_dim / 256;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int row = 0; row < out_dim; ++row) {
        float lanes[32];
        for (int lane = 0; lane < 32; ++lane) {
            float sum = 0.0f;
            for (int b = lane; b < nb; b += 32) {
                const uint8_t* blk = w + ((size_t)row * nb + b) * 56;
                const float d = hqo_half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
                if (isnan(d) || isinf(d)) continue;
                const float* xp = x + (size_t)b * 256;
                for (int by = 0; by < 50; ++by) {
                    uint32_t val = blk[2 + by];
                    for (int s = 0; s < 5; ++s) {
                        const int trit = (int)(val % 3) - 1;
                        val /= 3;
                        sum = fmaf(d * (float)trit, xp[by * 5 + s], sum);
                    }
                }
                for (int by = 50; by < 52; ++by) {
                    uint32_t val = blk[2 + by];
                    for (int s = 0; s < 3; ++s) {
                        const int trit = (int)(val % 3) - 1;
                        val /= 3;
                        sum = fmaf(d * (float)trit, xp[250 + (by - 50) * 3 + s], sum);
                    }
                }
            }
            lanes[lane] = sum;
        }
        for (int off = 16; off > 0; off /= 2) {
            float nxt[32];
            for (int i = 0; i < 32; ++i) nxt[i] = lanes[i] + (i + off < 32 ? lanes[i + off] : lanes[i]);
            memcpy(lanes, nxt, sizeof lanes);
        }
        out[row] = lanes[0];
    }
    return 0;
}

/* ------------------------------------------------- output / embedding */

static void warp_tree(float lanes[32]) {  /* forward_baseline.cu:42-48 */
    for (int off = 16; off > 0; off /= 2) {
        float nxt[32];
        for (int i = 0; i < 32; ++i) nxt[i] = lanes[i] + (i + off < 32 ? lanes[i + off] : lanes[i]);
        memcpy(lanes, nxt, 32 * sizeof(float));
    }
}

static int tq1_trit(const uint8_t* blk, int e) {  /* element e of a TQ1_0 block, native_decoder.cu:81-101 */
    uint32_t val;
    int s;
    if (e < 250) {
        val = blk[2 + e / 5];
        s = e % 5;
    } else {
        val = blk[2 + 50 + (e - 250) / 3];
        s = (e - 250) % 3;
    }
    for (int i = 0; i < s; ++i) val /= 3;
    return (int)(val % 3) - 1;
}

int hqo_output_projection(const float* x, const void* w, int type, float* logits,
                          int embedding_dim, int vocab_size, int nthreads) {
    const int K = embedding_dim;
    if (!x || !w || !logits || K <= 0 || vocab_size <= 0) return HQO_EINVAL;
    const int tq1 = type == HQO_GGML_TQ1_0 || type == HQO_GGML_TQ1_0_ALT;
    if (type != HQO_GGML_F32 && type != HQO_GGML_BF16 && type != HQO_GGML_Q8_0 && !tq1) return HQO_EINVAL;
    if ((type == HQO_GGML_Q8_0 && K % 32) || (tq1 && K % 256)) return HQO_EINVAL;
    nthreads = set_threads(nthreads);
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int row = 0; row < vocab_size; ++row) {
        float lanes[32];
        for (int lane = 0; lane < 32; ++lane) {
            float acc = 0.0f;
            if (type == HQO_GGML_F32) {
                const float* r = (const float*)w + (size_t)row * K;
                for (int i = lane; i < K; i += 32) acc = fmaf(r[i], x[i], acc);
            } else if (type == HQO_GGML_BF16) {
                const uint16_t* r = (const uint16_t*)w + (size_t)row * K;
                for (int i = lane; i < K; i += 32) {
                    const uint32_t u = (uint32_t)r[i] << 16;
                    float f;
                    memcpy(&f, &u, 4);
                    acc = fmaf(f, x[i], acc);
                }
            } else if (type == HQO_GGML_Q8_0) {
                const int nb = K / 32;
                const uint8_t* r = (const uint8_t*)w + (size_t)row * nb * 34;
                for (int b = lane; b < nb; b += 32) {
                    const uint8_t* blk = r + (size_t)b * 34;
                    const float d = hqo_half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
                    for (int j = 0; j < 32; ++j) acc = fmaf(d * (float)(int8_t)blk[2 + j], x[b * 32 + j], acc);
                }
            } else {
                const int nb = K / 256;
                const uint8_t* r = (const uint8_t*)w + (size_t)row * nb * 56;
                for (int b = 0; b < nb; ++b) {
                    const uint8_t* blk = r + (size_t)b * 56;
                    float d = hqo_half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
                    if (isnan(d) || isinf(d)) d = 0.0f;
                    for (int by = lane; by < 50; by += 32) {
                        uint32_t val = blk[2 + by];
                        for (int t = 0; t < 5; ++t) {
                            const int trit = (int)(val % 3) - 1;
                            val /= 3;
                            acc = fmaf(d * (float)trit, x[b * 256 + by * 5 + t], acc);
                        }
                    }
                    if (lane < 2) {
                        uint32_t val = blk[2 + 50 + lane];
                        for (int t = 0; t < 3; ++t) {
                            const int trit = (int)(val % 3) - 1;
                            val /= 3;
                            acc = fmaf(d * (float)trit, x[b * 256 + 250 + lane * 3 + t], acc);
                        }
                    }
                }
            }
            lanes[lane] = acc;
        }
        warp_tree(lanes);
        logits[row] = lanes[0];
    }
    return 0;
}

int hqo_embedding_lookup(const void* table, int type, int token_id, float* out, int embedding_dim) {
    const int K = embedding_dim;
    if (!table || !out || K <= 0 || token_id < 0) return HQO_EINVAL;
    const int tq1 = type == HQO_GGML_TQ1_0 || type == HQO_GGML_TQ1_0_ALT;
    if ((type == HQO_GGML_Q8_0 && K % 32) || (tq1 && K % 256)) return HQO_EINVAL;
    for (int i = 0; i < K; ++i) {
        if (type == HQO_GGML_F32) {
            out[i] = ((const float*)table)[(size_t)token_id * K + i];
        } else if (type == HQO_GGML_BF16) {
            const uint32_t u = (uint32_t)((const uint16_t*)table)[(size_t)token_id * K + i] << 16;
            memcpy(&out[i], &u, 4);
        } else if (type == HQO_GGML_Q8_0) {
            const uint8_t* blk = (const uint8_t*)table + ((size_t)token_id * (K / 32) + i / 32) * 34;
            const float d = hqo_half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
            out[i] = d * (float)(int8_t)blk[2 + i % 32];
        } else if (tq1) {
            const uint8_t* blk = (const uint8_t*)table + ((size_t)token_id * (K / 256) + i / 256) * 56;
            float d = hqo_half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
            if (isnan(d) || isinf(d)) d = 0.0f;
            out[i] = d * (float)tq1_trit(blk, i % 256);
        } else {
            return HQO_EINVAL;
        }
    }
    return 0;
}

/* ------------------------------------------------------------ W8A8 (int8) */

static int8_t q8_of(float x) {
    const float v = fminf(fmaxf(x * 127.0f, -128.0f), 127.0f);
    return (int8_t)v; /* truncation toward zero */
}

int hqo_w8_gemm(const float* X, const int8_t* W, const float* scales, float* Y,
                int M, int K, int N, int nthreads) {
    if (!X || !W || !scales || !Y || M < 0 || K <= 0 || N <= 0) return HQO_EINVAL;
    nthreads = set_threads(nthreads);
    const int quads = K / 4;
    #pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int m = 0; m < M; ++m) {
        int8_t* xq = (int8_t*)malloc((size_t)quads * 4);
        for (int k = 0; k < quads * 4; ++k) xq[k] = q8_of(X[(size_t)m * K + k]);
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int q = 0; q < quads; ++q) {
                int dot = 0;
                for (int i = 0; i < 4; ++i) dot += (int)xq[4 * q + i] * (int)W[(size_t)(4 * q + i) * N + n];
                acc = fmaf((float)dot, 1.0f / 127.0f, acc);
            }
            Y[(size_t)m * N + n] = acc * scales[n];
        }
        free(xq);
    }
    return 0;
}
