// hq_internal.h -- internal (non-ABI) interfaces between the API layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hq {

enum class DType : int { F32 = 0, F16 = 1, BF16 = 2 };

struct GemmArgs {
    const void* A;
    DType a_dtype;
    const uint8_t* W;  // tile format
    int wbits;         // 4 or 2
    const void* S;
    DType s_dtype;
    const float* bias;  // nullable
    void* C;
    DType c_dtype;
    int M, N, K, group;
    bool weights_just_written;  // W was produced by the preceding kernel on the stream
    uint8_t* ws;  // 256-byte aligned workspace (after any re-tiled weights)
    size_t ws_bytes;
    cudaStream_t stream;
};

struct DeviceInfo {
    int sm_count;
    int cc_major, cc_minor;
    size_t smem_optin;
};
const DeviceInfo& device_info(int dev);
// Sets cudaFuncAttributeMaxDynamicSharedMemorySize once per (function, device).
cudaError_t ensure_smem_attr(const void* fn, int dev, int bytes);
// Clusters of `cs` CTAs of `fn` (threads, dynamic smem) that can be resident at
// once on device `dev` (cached; cs > 8 enables non-portable cluster sizes on fn).
// 0 when such a cluster cannot be launched.
int max_active_clusters(const void* fn, int threads, int smem, int cs, int dev);

// Decode (M <= 16) HBM-streaming kernels.  The workspace holds, for the
// integer-MMA kernel only, per-strip-group arrival counters, the split
// partials and the activation pieces with their scales.
size_t decode_workspace_bytes(int M, int N, int K, int wbits, int dev);
// int4 codes x fp16/bf16 activations on the integer tensor cores (no bias).
bool decode_i8_supported(const GemmArgs& a);
size_t decode_i8_workspace_bytes(int N, int K, int dev);
cudaError_t launch_decode_i8(const GemmArgs& a, bool early_weights);
bool decode_supported(const GemmArgs& a);
// Programmatic dependent launch lets a decode GEMM stream its weights while the
// previous kernel on the stream finishes (on by default).
void set_decode_launch_overlap(bool on);
cudaError_t launch_decode(const GemmArgs& a);
// Decode on the tcgen05 tensor cores (16-bit activations and scales, no bias,
// group a multiple of 128); launch_decode dispatches to it when supported.
bool decode_tc_supported(const GemmArgs& a);
cudaError_t launch_decode_tc(const GemmArgs& a, bool early_weights);

// Tensor-core (tcgen05) kernel for larger M.
size_t prefill_workspace_bytes(int M, int N, int K, int wbits, int dev);
bool prefill_supported(const GemmArgs& a);
cudaError_t launch_prefill(const GemmArgs& a);

// Repack kernels (device).
// k32: the TILE_U4_K32 order (int4, group 32).
cudaError_t launch_linear_to_tile(const void* src, bool src_is_quad, int wbits, uint8_t* dst, int K, int N,
                                  cudaStream_t s, bool k32 = false);
cudaError_t launch_tile_to_linear(const uint8_t* src, int wbits, uint32_t* dst, int K, int N, cudaStream_t s,
                                  bool k32 = false);
cudaError_t launch_linear_to_quad(const uint32_t* src, uint32_t* dst, int K, int N, bool inverse, cudaStream_t s);
// GGUF Q4_K [N][K/256] blocks -> TILE_U4_K32 codes + f32 group-32 scales and biases [K/32][N].
cudaError_t launch_q4k_to_tile(const uint8_t* w, uint8_t* tile, float* scales, float* bias, int K, int N,
                               cudaStream_t s);

namespace host {
void linear_to_tile(const uint32_t* src, bool quad, int wbits, uint32_t* dst, int K, int N, int nthreads,
                    bool k32 = false);
void tile_to_linear(const uint32_t* src, int wbits, uint32_t* dst, int K, int N, int nthreads, bool k32 = false);
void linear_quad(const uint32_t* src, uint32_t* dst, int K, int N, bool inverse, int nthreads);
void q4k_to_tile(const uint8_t* w, uint32_t* tile, float* scales, float* bias, int K, int N, int nthreads);
}  // namespace host

// TQ1_0 kernels.
cudaError_t launch_tq1_0_gemv(const float* x, const uint8_t* w, float* out, int in_dim, int out_dim, cudaStream_t s);
cudaError_t launch_w8_gemm(const float* X, const int8_t* W, const float* scales, float* Y, int M, int K, int N,
                           cudaStream_t s);
cudaError_t launch_output_projection(const float* x, const uint8_t* w, int type, float* out, int K, int N,
                                     cudaStream_t s);
cudaError_t launch_embedding_lookup(const uint8_t* table, int type, int token_id, float* out, int K, cudaStream_t s);
cudaError_t launch_tq1_0_to_tile_t2(const uint8_t* w, uint8_t* tile, uint16_t* scales, int K, int N, cudaStream_t s);

// Plain fp32 GEMM (the engine shim's forward_reference).
cudaError_t launch_f32_gemm(const float* X, const float* W, float* Y, int M, int K, int N, cudaStream_t s);
// Scalar int4 GEMM on the linear layout (the engine shim's forward_baseline_int4); B may be null.
cudaError_t launch_baseline_u4(const float* X, const uint32_t* W, const float* S, const float* B, float* Y, int M,
                               int K, int N, int group, cudaStream_t s);

// Message returned by hq_last_error_string() on this host thread.
void set_last_error(const char* msg);

// Device error word: address on device `dev` (passed to kernels), read+clear.
unsigned* device_error_word(int dev);
cudaError_t read_and_clear_device_error(unsigned* code);

}  // namespace hq
