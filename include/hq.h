/*
 * hq.h -- C ABI of the B200 (sm_100a) quantized-linear library (libhq.so).
 *
 * Drop-in replacement for the quantized linear layer of the hydrogen engine:
 * int4 (W4A16) and ternary packed weights times fp16/bf16 activations with
 * fp32 accumulation.  Every entry point is plain C: device pointers, sizes,
 * enums and a CUDA stream handle; no exceptions cross this boundary.
 *
 * Reference interfaces replaced (paths inside the Nebula project):
 *   hydrogen/include/marlin_gemm.hpp:59-172   hydrogen::MarlinGemmEngine
 *   hydrogen/src/model/marlin_gemm.cu:432-467 repack_q4k_to_marlin (host repack)
 *   hydrogen/src/model/marlin_gemm.cu:556-601 forward_marlin_int4 (the GEMM launch)
 *   hydrogen/src/model/native_decoder.cu:155-206 kernel_gemv_tq1_0 (ternary GEMV)
 * The reference has no C ABI for this path (its Rust crate
 * crates/nebula-hydrogen exports IPC types only); these functions are additive.
 *
 * Conventions
 *   - All tensor arguments are device pointers unless the name says host.
 *   - Row-major: A is [M][K] (lda = K), C is [M][N] (ldc = N), scales and
 *     biases are [K/group][N] (marlin_gemm.hpp:161-162).
 *   - Device pointers handed to hq_gemm are 16-byte aligned.
 *   - Calls are asynchronous on `stream`, stream-ordered, allocate nothing,
 *     and may run concurrently on different streams with different
 *     workspaces.  C is overwritten.
 *   - Shapes: N % 16 == 0, K % 64 == 0, group == 32 or group % 64 == 0,
 *     K % group == 0 (the reference needs K % 512 == 0 and group % 32 == 0:
 *     marlin_gemm.cu:156-159, so every reference shape with group 32 or a
 *     multiple of 64 is accepted).  Group 32 takes int4 weights in
 *     HQ_WFMT_TILE_U4_K32 (or a reference layout, re-tiled into it) with f32
 *     scales: M <= 16 runs on the split-K decode kernel (two scale and bias
 *     rows per 64-k block), larger M on the tcgen05 kernel.
 */
#ifndef HQ_H
#define HQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define HQ_API __declspec(dllexport)
#else
#define HQ_API __attribute__((visibility("default")))
#endif

/* Same object as cudaStream_t; declared here so callers need no CUDA headers. */
typedef struct CUstream_st* hq_stream_t;

typedef enum hq_status {
    HQ_OK = 0,
    HQ_ERR_INVALID_ARG = 1,       /* null pointer, bad enum, negative size */
    HQ_ERR_UNSUPPORTED_SHAPE = 2, /* shape outside the rules above */
    HQ_ERR_WORKSPACE_TOO_SMALL = 3,
    HQ_ERR_CUDA = 4,              /* a CUDA runtime call failed; see hq_last_error_string */
    HQ_ERR_TIMEOUT = 5,           /* a bounded device-side wait gave up */
    HQ_ERR_MISALIGNED = 6,        /* a pointer breaks the 16-byte alignment rule */
    HQ_ERR_UNSUPPORTED_DEVICE = 7 /* not an sm_100 device */
} hq_status;

typedef enum hq_dtype { HQ_F32 = 0, HQ_F16 = 1, HQ_BF16 = 2 } hq_dtype;

typedef enum hq_wfmt {
    /* uint32 [K/8][N]; word (kw,n) holds k = 8kw+i at bits 4i, code u = q+8.
     * marlin_gemm.cu:495-510 (the reference's "linear" layout). */
    HQ_WFMT_LINEAR_U4 = 0,
    /* uint4 [K/32][N]; quad (kq,n) word j = linear word (4kq+j, n).
     * marlin_gemm.cu:446-455 (the reference's "Marlin" layout). */
    HQ_WFMT_MARLIN_QUAD = 1,
    /* This library's tile order for int4: 16 columns x 64 k chunks of 512
     * bytes, each lane's 16 bytes ready for one register dequant; strip
     * groups of 128 columns contiguous along k.  Produced by hq_repack_*. */
    HQ_WFMT_TILE_U4 = 2,
    /* uint32 [K/16][N]; word (kw,n) holds k = 16kw+i at bits 2i, code t+1. */
    HQ_WFMT_LINEAR_T2 = 3,
    /* Tile order for 2-bit ternary (256-byte chunks). */
    HQ_WFMT_TILE_T2 = 4,
    /* [N][K/256] blocks of 56 bytes {fp16 d; u8 packed[52]; u16 pad}
     * (native_decoder.cu:32-36). */
    HQ_WFMT_TQ1_0 = 5,
    /* TILE_U4 for scale groups of 32 k: lane t's two words per column hold
     * k 8t..8t+7 and 32+8t..32+8t+7 of each 64-k block, so every MMA step stays
     * inside one scale group.  hq_gemm takes group 32 only in this layout (or
     * from LINEAR_U4 / MARLIN_QUAD, re-tiled into it). */
    HQ_WFMT_TILE_U4_K32 = 6
} hq_wfmt;

/* Library version string, e.g. "hq 0.1.0 sm_100a". */
HQ_API const char* hq_version(void);

/* Message for the most recent failing call on this host thread. */
HQ_API const char* hq_last_error_string(void);

/* Bytes of a packed weight tensor in `fmt` (0 if the shape is invalid). */
HQ_API size_t hq_weight_bytes(hq_wfmt fmt, int K, int N);

/* Workspace bytes that hq_gemm needs for this problem (a multiple of 256;
 * 0 when none is needed, in which case workspace may be NULL).  The workspace
 * holds re-tiled weights for the reference layouts and the decode kernel's
 * split state: one arrival counter per 128-column group and the fp32 partial
 * tiles of groups shared by two SMs.  Zero-fill it once before first use
 * (hq_workspace_init); every call leaves the counters at zero again, so no
 * per-call memset.  A call that fails with HQ_ERR_TIMEOUT may leave counters
 * set: zero-fill again before the next call.  One workspace per stream: calls
 * that may run at the same time need different workspaces. */
HQ_API size_t hq_gemm_workspace_size(int M, int N, int K, int group, hq_wfmt wfmt);
HQ_API hq_status hq_workspace_init(void* workspace, size_t ws_bytes, hq_stream_t stream);

/*
 * The quantized linear layer:  C[M][N] = A[M][K] * dequant(Wq)   (fp32 accumulate)
 *   dequant: int4   w = (u - 8) * scale[g][n]            (bias == NULL)
 *                   w = u * scale[g][n] + bias[g][n]     (bias != NULL; reference
 *                                                          form, marlin_gemm.cu:208-209)
 *            ternary w = t * scale[g][n]
 *   a_dtype: HQ_F16 | HQ_BF16 | HQ_F32.  f32 activations keep ~fp32 accuracy:
 *            held on chip as two fp16 terms or, at M <= 4, as two fixed-point
 *            parts of 15 bits per (token, scale group), 30 bits in all.  At
 *            M <= 4 on layers of >= 16384 columns, 16-bit activations are held
 *            as one 15-bit fixed-point copy per (token, scale group): the
 *            result stays within ~1e-5 of max|C| of the fp32 product.  A scale
 *            group of activations holding Inf/NaN makes that token's outputs NaN.
 *   s_dtype: HQ_F16 | HQ_BF16 | HQ_F32; bias is always f32.  Combinations
 *            (activations, scales): (f16, f16), (bf16, bf16), (f16 | bf16 | f32,
 *            f32), (f32, f16); a bias goes with f32 scales and f16 / f32
 *            activations.  Group 32: f32 scales only.  Ternary weights:
 *            (f16, f16), (bf16, bf16), (f32, f16) (the last with f32 output:
 *            TQ1_0 layers converted by hq_tq1_0_to_tile_t2, fp32 x as in
 *            kernel_gemv_tq1_0).
 *   c_dtype: HQ_F16 | HQ_BF16 | HQ_F32: the activation type, or f32
 *   wfmt:    HQ_WFMT_TILE_U4 (groups that are multiples of 64),
 *            HQ_WFMT_TILE_U4_K32 (group 32) and HQ_WFMT_TILE_T2 run directly.
 *            LINEAR_U4, MARLIN_QUAD and LINEAR_T2 are accepted for drop-in use
 *            and are re-tiled into the workspace first (one extra pass over
 *            the weights); hq_gemm_workspace_size accounts for it.
 * M <= 16 runs the HBM-streaming decode kernel; larger M runs the tcgen05
 * tensor-core kernel, which rounds each dequantised weight to the 16-bit
 * activation type (with f32 scales: u * s + b formed in fp32, rounded once).
 * f32 activations at M > 16 run the decode kernel 16 rows per launch.
 * Launch overlap (on by default, see hq_set_launch_overlap): a call may start
 * reading Wq and scales while the kernel enqueued just before it on the same
 * stream is still running (programmatic dependent launch); A is read only
 * after that kernel has finished.  Tile-order weights must therefore not be
 * written by the immediately preceding kernel on the stream (weights loaded at
 * start-up, as in the hydrogen engine, are fine); reference-layout weights
 * (re-tiled inside the call) are never read early.
 * Replaces MarlinGemmEngine::forward_marlin_int4 (marlin_gemm.cu:556-601).
 */
HQ_API hq_status hq_gemm(const void* A, hq_dtype a_dtype,
                         const void* Wq, hq_wfmt wfmt,
                         const void* scales, hq_dtype s_dtype,
                         const float* bias,
                         void* C, hq_dtype c_dtype,
                         int M, int N, int K, int group,
                         void* workspace, size_t ws_bytes,
                         hq_stream_t stream);

/* Size of the scratch array that hq_gemm_noalloc uses in place of a workspace. */
#define HQ_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/*
 * hq_gemm for callers that cannot allocate device memory, e.g. a plugin
 * inside a serving process that owns and budgets every byte of device memory
 * (a pre-sized arena or another framework's allocator), where an extra
 * cudaMalloc is not allowed or would stall the device mid-step.  Same
 * arguments and results as hq_gemm minus the workspace: the workspace is a
 * HQ_NOALLOC_SCRATCH_BYTES array compiled into this library.  This entry
 * point allocates nothing and calls no allocating routine.
 *   - Limit: a problem whose hq_gemm_workspace_size exceeds
 *     HQ_NOALLOC_SCRATCH_BYTES fails with HQ_ERR_WORKSPACE_TOO_SMALL (reference
 *     layouts need K*N/2 bytes for int4, K*N/4 for ternary, plus the decode
 *     kernel's split state of about 2.4 MB on a 148-SM B200).
 *   - The first call on a device that needs scratch, with that device
 *     current, looks up the array's device address, zero-fills it and waits
 *     for the device (cudaDeviceSynchronize); make that first call before any
 *     stream capture.
 *   - The array is part of the library's device code: it occupies
 *     HQ_NOALLOC_SCRATCH_BYTES on every device where the library's module is
 *     loaded (from the first call under lazy module loading, the CUDA default;
 *     from context creation with CUDA_MODULE_LOADING=EAGER) until the process
 *     exits.
 *   - All calls on a device share the array, which keeps the previous call's
 *     contents; calls whose GPU work overlaps (different streams, several host
 *     threads) race on it, so keep them on one stream.
 * No counterpart in the reference: it exists only for the callers above.
 */
HQ_API hq_status hq_gemm_noalloc(const void* A, hq_dtype a_dtype,
                                 const void* Wq, hq_wfmt wfmt,
                                 const void* scales, hq_dtype s_dtype,
                                 const float* bias,
                                 void* C, hq_dtype c_dtype,
                                 int M, int N, int K, int group,
                                 hq_stream_t stream);

/*
 * Weight repack between formats, bit-exact in both directions.
 * Supported (src -> dst): LINEAR_U4 -> MARLIN_QUAD (the reference repack,
 * marlin_gemm.cu:432-467), MARLIN_QUAD -> LINEAR_U4, LINEAR_U4 -> TILE_U4
 * and TILE_U4_K32, MARLIN_QUAD -> TILE_U4 and TILE_U4_K32, TILE_U4 and
 * TILE_U4_K32 -> LINEAR_U4, LINEAR_T2 -> TILE_T2, TILE_T2 -> LINEAR_T2.
 * hq_repack_host takes host pointers and runs synchronously on host threads
 * (replaces MarlinGemmEngine::repack_q4k_to_marlin, marlin_gemm.hpp:78-83);
 * hq_repack_device takes device pointers and runs on `stream`.
 */
HQ_API hq_status hq_repack_host(const void* src, hq_wfmt src_fmt, void* dst, hq_wfmt dst_fmt,
                                int K, int N, int nthreads);
HQ_API hq_status hq_repack_device(const void* src, hq_wfmt src_fmt, void* dst, hq_wfmt dst_fmt,
                                  int K, int N, hq_stream_t stream);

/*
 * TQ1_0 matrix-vector product in the reference's own layout:
 *   out[row] = sum_b sum_j d_b * trit_j * x[256b + j]; blocks with NaN/Inf d
 *   are skipped.  x, out fp32; w = [out_dim][in_dim/256] TQ1_0 blocks.
 * Replaces kernel_gemv_tq1_0 (native_decoder.cu:155-206), computing every row.
 * in_dim % 1024 == 0 with w 16-byte aligned takes the tensor-core kernel (x as
 * a 28-bit fixed-point copy relative to max|x|: results within 1e-5 of max|out|
 * of the fp32 loop, deterministic); other shapes, and any x holding NaN/Inf,
 * take the fp32 loop.  Requires w 8-byte and x 4-byte aligned.
 */
HQ_API hq_status hq_tq1_0_gemv(const float* x, const void* w, float* out,
                               int in_dim, int out_dim, hq_stream_t stream);

/*
 * Offline conversion of TQ1_0 weights ([N][K/256] blocks) into TILE_T2 codes
 * plus fp16 group-128 scales [K/128][N] (the block scale repeated for both
 * halves; a NaN/Inf block scale becomes 0, matching the reference's skip).
 */
HQ_API hq_status hq_tq1_0_to_tile_t2(const void* w_tq1, void* tile_t2, void* scales_f16,
                                     int K, int N, hq_stream_t stream);

/*
 * Model-load conversion of GGUF Q4_K weights (type 12: 256 weights per 144-byte
 * block, gguf_parser.hpp:44,130; laid out [N][K/256] as the native decoder maps
 * GGUF tensors, native_decoder.cu:849-918) into TILE_U4_K32 codes plus f32
 * group-32 scales and biases [K/32][N].  The block fields follow llama.cpp's
 * block_q4_K: fp16 d and dmin, 6-bit scale sc_i and min m_i per 32 weights,
 * 4-bit codes u.  Then hq_gemm(A, a, tile, HQ_WFMT_TILE_U4_K32, scales, HQ_F32,
 * bias, C, c, M, N, K, 32, ...) computes with w = u * (d sc_i) - dmin m_i,
 * llama.cpp's dequantize_row_q4_K; scale and bias are exact in f32.
 * K % 256 == 0, N % 16 == 0; w_q4k 8-byte aligned, the outputs 4-byte aligned.
 * The _host form runs on host threads (nthreads <= 0: all) with host pointers.
 */
HQ_API hq_status hq_q4_k_to_tile(const void* w_q4k, void* tile, float* scales, float* bias,
                                 int K, int N, hq_stream_t stream);
HQ_API hq_status hq_q4_k_to_tile_host(const void* w_q4k, void* tile, float* scales, float* bias,
                                      int K, int N, int nthreads);

/*
 * W8A8 GEMM, the reference engine's third precision: activations quantized per
 * element as q8(x) = (int8) trunc(clamp(x * 127, -128, 127)), int8 weights
 * W [K][N] (k-major rows), one fp32 scale per column:
 *   Y[m][n] = scale[n] * sum over the K/4 whole quads of k of q8(X[m][k]) W[k][n] / 127.
 * Replaces MarlinGemmEngine::forward_cutlass_int8 / kernel_cutlass_int8_gemm
 * (marlin_gemm.cu:327-377, 603-617); any M (the reference's acc[8] stops at 8).
 * The int32 sums are exact and rounded once (the reference rounds an fp32
 * running sum per quad): results within 1e-5 of max|Y| of the reference's.
 * N % 4 == 0, K <= 65536, W 4-byte aligned.  One launch per 8 rows of X.
 */
HQ_API hq_status hq_w8_gemm(const float* X, const int8_t* W, const float* scales, float* Y,
                            int M, int K, int N, hq_stream_t stream);

/* GGML tensor type ids of the projection weights (gguf_parser.hpp:33-64). */
#define HQ_GGML_F32 0
#define HQ_GGML_Q8_0 8
#define HQ_GGML_BF16 30
#define HQ_GGML_TQ1_0 34
#define HQ_GGML_TQ1_0_ALT 143 /* read as TQ1_0, as forward_baseline.cu:82,218 do */

/*
 * Output projection: logits[row] = dot(W[row, :], x), fp32 x [embedding_dim],
 * fp32 logits [vocab_size].  W rows by w_type: HQ_GGML_F32 / HQ_GGML_BF16
 * embedding_dim elements; HQ_GGML_Q8_0 embedding_dim/32 blocks of 34 bytes
 * (fp16 d + 32 int8, d applied unchecked); HQ_GGML_TQ1_0 (or _ALT)
 * embedding_dim/256 TQ1_0 blocks, computed by hq_tq1_0_gemv.
 * Replaces kernel_output_projection (forward_baseline.cu:178-257) and its
 * launch (:489-499).  Fast paths: F32 with embedding_dim % 4 == 0 and W
 * 16-byte aligned, BF16 with embedding_dim % 8 == 0 and W 16-byte aligned,
 * Q8_0 with embedding_dim % 64 == 0 and W 4-byte aligned; other shapes run the
 * reference's own lane loop.  x 4-byte aligned.  No workspace.
 */
HQ_API hq_status hq_output_projection(const float* x, const void* w, int w_type, float* logits,
                                      int embedding_dim, int vocab_size, hq_stream_t stream);

/*
 * Embedding row lookup: out[i] = W[token_id, i] as fp32 (Q8_0: d * q; TQ1_0:
 * d * trit with a NaN/Inf d read as 0).  Replaces kernel_embedding_lookup
 * (forward_baseline.cu:55-109; native_decoder.cu:63-103 for TQ1_0).  Adds
 * vocab_size, only to reject token_id outside [0, vocab_size) -- the reference
 * reads out of bounds there.
 */
HQ_API hq_status hq_embedding_lookup(const void* table, int w_type, int token_id, float* out,
                                     int embedding_dim, int vocab_size, hq_stream_t stream);

/*
 * In-place sum over the `world` GPUs of one node (tensor-parallel all-reduce of
 * the row-parallel GEMM outputs), through peer memory over NVLink.
 *   peer_bufs[j]:  rank j's buffer of `count` HQ_BF16 / HQ_F16 elements, as
 *                  addressable from this GPU (peer-mapped memory, e.g. PyTorch
 *                  symmetric memory); host array of `world` device addresses.
 *   peer_flags[j]: rank j's flag area, 32 zero-initialised uint32 (peer-mapped).
 *   multicast:     NVLink multicast (NVLS) address of the buffers, or NULL.  With
 *                  it the switch sums (multimem.ld_reduce, fp32 accumulation)
 *                  and broadcasts (multimem.st): each rank moves 2/world of the
 *                  vector over NVLink instead of 2 (world-1)/world.
 *   epoch:         1 for the first call on these flags, +1 for every call after;
 *                  or 0 on every call: the kernel then takes the same number
 *                  from a call counter in the flag area, so the call can be
 *                  captured in a CUDA graph and replayed.
 *   ctas:          CTAs per call (the same on every call with these flags).
 * Every rank makes the same calls in the same order on its own stream; on
 * return every buffer holds the sum (fp32 accumulation; every rank holds the
 * same bits: in rank order 0..world-1 without multicast, in the switch's order
 * with it).  Waits for peers are bounded: a rank that never
 * arrives makes the others record HQ_ERR_TIMEOUT (hq_check_device_error).
 * No counterpart in the reference (it has no multi-GPU path).
 */
HQ_API hq_status hq_allreduce_sum(void* const* peer_bufs, unsigned* const* peer_flags, void* multicast,
                                  int world, int rank, hq_dtype dtype, size_t count, unsigned epoch, int ctas,
                                  hq_stream_t stream);

/* Turn the launch overlap described at hq_gemm on (1, default) or off (0)
 * for the whole process. */
HQ_API void hq_set_launch_overlap(int enable);

/*
 * Device-side error word: kernels that wait on barriers give up after a
 * bounded time and record a code here instead of hanging.  Synchronises the
 * current device, returns HQ_ERR_TIMEOUT (and clears the word) if any kernel
 * recorded a timeout since the last call, else HQ_OK.
 */
HQ_API hq_status hq_check_device_error(void);

/*
 * C wrappers of the drop-in hydrogen::MarlinGemmEngine shim
 * (include/hq_marlin_gemm.hpp), for callers without C++.
 * Same arguments and meaning as marlin_gemm.hpp:61, :78-83, :88-95, :100-107,
 * :123-128, :133-139.  Return HQ_OK or an error code instead of throwing.
 */
typedef struct hq_marlin_engine hq_marlin_engine;
HQ_API hq_marlin_engine* hq_marlin_engine_create(uint32_t M, uint32_t K, uint32_t N, uint32_t group_size);
HQ_API void hq_marlin_engine_destroy(hq_marlin_engine* e);
HQ_API hq_status hq_marlin_repack_q4k_to_marlin(hq_marlin_engine* e, const uint8_t* h_src_q4k,
                                                uint32_t* h_dst_marlin, uint32_t K, uint32_t N,
                                                double* repack_ms);
HQ_API hq_status hq_marlin_forward_marlin_int4(hq_marlin_engine* e, const float* d_X,
                                               const uint32_t* d_W_marlin, const float* d_scales,
                                               const float* d_biases, float* d_Y, uint32_t M);
HQ_API hq_status hq_marlin_forward_baseline_int4(hq_marlin_engine* e, const float* d_X,
                                                 const uint32_t* d_W_linear, const float* d_scales,
                                                 const float* d_biases, float* d_Y, uint32_t M);
HQ_API hq_status hq_marlin_forward_reference(hq_marlin_engine* e, const float* d_X,
                                             const float* d_W_dequant, float* d_Y_ref, uint32_t M);
HQ_API hq_status hq_marlin_forward_cutlass_int8(hq_marlin_engine* e, const float* d_X,
                                                const int8_t* d_W_int8, const float* d_scales,
                                                float* d_Y, uint32_t M);
HQ_API hq_status hq_marlin_verify_fidelity(hq_marlin_engine* e, const float* d_Y_ref,
                                           const float* d_Y_marlin, uint32_t M,
                                           double* max_abs_err, double* mse);

/* ------------------------------------------------------ split-fuse batching
 * Replaces hydrogen::SplitFuseBatcher (batcher.hpp:98-199, split_fuse.cpp):
 * same request life cycle and step assembly; hq_batcher_execute runs the step
 * through real hq_gemm layers where the reference's execute_step
 * (split_fuse.cpp:196-238) simulates it.  Host-side object, not thread-safe. */
typedef struct hq_batcher hq_batcher;

/* RequestStatus (batcher.hpp:17-22). */
enum { HQ_REQ_QUEUED = 0, HQ_REQ_RUNNING_PREFILL = 1, HQ_REQ_RUNNING_DECODE = 2, HQ_REQ_COMPLETED = 3 };

/* SplitFuseConfig (batcher.hpp:66-74): the scheduling fields. */
typedef struct hq_batcher_config {
    uint32_t max_prefill_chunk_tokens; /* 64 in the reference */
    uint32_t max_decode_streams;       /* 16: a sizing hint, not enforced (as in the reference) */
    uint32_t max_batch_tokens;         /* 512 */
} hq_batcher_config;

/* BatchChunk (batcher.hpp:40-45). */
typedef struct hq_batch_chunk {
    uint32_t request_id, start_token, num_tokens;
    int is_prefill;
} hq_batch_chunk;

/* FusedBatch's counters (batcher.hpp:50-56). */
typedef struct hq_batch_info {
    uint32_t num_decode_requests, num_prefill_tokens, total_batch_tokens;
    double assembly_overhead_us;
} hq_batch_info;

typedef struct hq_request_state {
    uint32_t prompt_tokens, prefill_completed_tokens, decode_tokens_generated, max_decode_tokens;
    int status;
} hq_request_state;

/* One quantized linear layer of the stack a step runs through. */
typedef struct hq_linear_layer {
    const void* W;
    hq_wfmt wfmt;
    const void* scales;
    hq_dtype s_dtype;
    const float* bias; /* nullable */
    int K, N, group;
} hq_linear_layer;

/* cfg NULL: the reference's defaults (64, 16, 512). */
HQ_API hq_batcher* hq_batcher_create(const hq_batcher_config* cfg);
HQ_API void hq_batcher_destroy(hq_batcher* b);
HQ_API void hq_batcher_reset(hq_batcher* b);
/* submit_request: returns the new request id (1, 2, ...). */
HQ_API uint32_t hq_batcher_submit(hq_batcher* b, uint32_t prompt_tokens, uint32_t max_decode_tokens);
/* assemble_step_batch: writes the step's chunks (decode rows first, then at
 * most one prefill chunk) and returns their count, or -1 when max_chunks is
 * too small (active decode streams + 1 always suffices). */
HQ_API int hq_batcher_assemble(hq_batcher* b, hq_batch_chunk* chunks, int max_chunks, hq_batch_info* info);
/* update_step_completion. */
HQ_API hq_status hq_batcher_complete(hq_batcher* b, const hq_batch_chunk* chunks, int n);
HQ_API int hq_batcher_has_work(const hq_batcher* b);
HQ_API size_t hq_batcher_active_requests(const hq_batcher* b);
HQ_API hq_status hq_batcher_request_state(const hq_batcher* b, uint32_t request_id, hq_request_state* out);
/* Runs `rows` activation rows (the step's total_batch_tokens) through the
 * layers in order with hq_gemm: layer i reads act0 (i even) or act1 as a
 * contiguous [rows][K] array and writes the other as [rows][N]; each buffer
 * holds rows x max(K, N) elements of a_dtype; layer i+1's K must be layer i's
 * N; one zero-initialised workspace of hq_gemm_workspace_size for the largest
 * layer at M = rows serves every layer (the calls are stream-ordered).  The
 * result is in act1 for an odd number of layers, in act0 otherwise. */
HQ_API hq_status hq_batcher_execute(hq_batcher* b, uint32_t rows, const hq_linear_layer* layers, int n_layers,
                                    void* act0, void* act1, hq_dtype a_dtype, void* workspace, size_t ws_bytes,
                                    hq_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HQ_H */
