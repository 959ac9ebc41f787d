// hq_marlin_gemm.hpp -- source-compatible drop-in for hydrogen/include/marlin_gemm.hpp.
//
// Same namespace, types and public methods as the reference's
// hydrogen::MarlinGemmEngine (marlin_gemm.hpp:13-172); the work is done by
// libhq.so's sm_100a kernels through the C ABI in hq.h.  Semantics kept:
// device-pointer arguments, fp32 X / scales / biases / Y, w = u*scale + bias,
// Y overwritten, asynchronous on the legacy default stream, std::runtime_error
// on a CUDA failure.  Differences (documented, deliberate):
//   * Marlin-quad weights handed to forward_marlin_int4 are re-tiled on
//     device into an engine-owned buffer on every call; hq_repack_* + hq_gemm
//     on tile-order weights skip that pass;
//   * M up to any value (the reference silently overflows for M > 8,
//     marlin_gemm.cu:260,304);
//   * bandwidth_utilization_pct is relative to kPeakBandwidthGBs (B200
//     nominal HBM3e) instead of the RTX 4070's 504 GB/s (:677);
//   * forward_cutlass_int8 sums the dp4a products exactly in int32 and rounds
//     once (the reference rounds an fp32 running sum per 4 k), any M.
// forward_baseline_int4 keeps the reference's role: an un-optimised scalar
// kernel on the linear layout, the comparator of run_benchmark_sweep's
// speedup_ratio (use forward_marlin_int4 or hq_gemm for speed).
// The class is exported from libhq.so, so a program written against the
// reference header links against it unchanged.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace hydrogen {

struct MarlinGemmConfig {
    uint32_t M = 8;
    uint32_t K = 4096;
    uint32_t N = 4096;
    uint32_t group_size = 128;
};

struct MarlinBenchmarkResult {
    uint32_t M = 1;
    uint32_t K = 4096;
    uint32_t N = 4096;
    float marlin_latency_ms = 0.0f;
    float baseline_latency_ms = 0.0f;
    double marlin_tflops = 0.0;
    double marlin_bandwidth_gbs = 0.0;
    double bandwidth_utilization_pct = 0.0;
    double speedup_ratio = 1.0;
    double max_abs_error = 0.0;
    double mean_squared_error = 0.0;
    bool numerical_match = true;
    bool latency_target_met = true;
    bool bandwidth_target_met = true;
};

struct MarlinRepackResult {
    size_t num_weights = 0;
    double repack_time_ms = 0.0;
    double repack_time_seconds = 0.0;
    bool repack_under_1s = true;
};

class __attribute__((visibility("default"))) MarlinGemmEngine {
public:
    static constexpr double kPeakBandwidthGBs = 7700.0;

    explicit MarlinGemmEngine(MarlinGemmConfig config);
    ~MarlinGemmEngine();

    MarlinGemmEngine(const MarlinGemmEngine&) = delete;
    MarlinGemmEngine& operator=(const MarlinGemmEngine&) = delete;
    MarlinGemmEngine(MarlinGemmEngine&&) = delete;
    MarlinGemmEngine& operator=(MarlinGemmEngine&&) = delete;

    MarlinRepackResult repack_q4k_to_marlin(const uint8_t* h_src_q4k, uint32_t* h_dst_marlin, uint32_t K,
                                            uint32_t N);

    void forward_baseline_int4(const float* d_X, const uint32_t* d_W_linear, const float* d_scales,
                               const float* d_biases, float* d_Y, uint32_t M);

    void forward_marlin_int4(const float* d_X, const uint32_t* d_W_marlin, const float* d_scales,
                             const float* d_biases, float* d_Y, uint32_t M);

    void forward_reference(const float* d_X, const float* d_W_dequant, float* d_Y_ref, uint32_t M);

    // W8A8 path (marlin_gemm.hpp:112-118): int8 W [K][N], per-column fp32 scale.
    void forward_cutlass_int8(const float* d_X, const int8_t* d_W_int8, const float* d_scales, float* d_Y, uint32_t M);

    void verify_fidelity(const float* d_Y_ref, const float* d_Y_marlin, uint32_t M, double& out_max_abs_err,
                         double& out_mse);

    std::vector<MarlinBenchmarkResult> run_benchmark_sweep(int warmups = 5, int iterations = 20);

    MarlinRepackResult benchmark_repacking();

    [[nodiscard]] const MarlinGemmConfig& config() const noexcept { return config_; }

private:
    MarlinGemmConfig config_;
    void* d_workspace_{nullptr};
    size_t workspace_bytes_{0};
    // Synthetic data for run_benchmark_sweep (allocated on first use).
    float* d_X_{nullptr};
    uint32_t* d_W_linear_{nullptr};
    uint32_t* d_W_marlin_{nullptr};
    float* d_scales_{nullptr};
    float* d_biases_{nullptr};
    float* d_W_dequant_{nullptr};
    float* d_Y_ref_{nullptr};
    float* d_Y_marlin_{nullptr};
    float* d_Y_baseline_{nullptr};

    void ensure_workspace(uint32_t M);
    void ensure_synthetic_data();
    void free_device_memory();
    void run(const float* d_X, const uint32_t* d_W, int wfmt, const float* d_scales, const float* d_biases,
             float* d_Y, uint32_t M);
};

}  // namespace hydrogen
