// hq_marlin_engine.cu -- hydrogen::MarlinGemmEngine drop-in (include/hq_marlin_gemm.hpp)
// on top of the C ABI, plus its C wrappers (hq_marlin_* in hq.h).
//
// Mirrors hydrogen/src/model/marlin_gemm.cu:381-758 method by method; the
// kernels are this library's (decode / tensor-core), the fp32 check GEMM is the
// bit-compatible restatement of kernel_reference_gemm (hq_misc.cu), and
// forward_baseline_int4 is, as in the reference, an un-optimised scalar kernel
// on the linear layout: the yardstick run_benchmark_sweep's speedup_ratio
// measures forward_marlin_int4 against.
#include "hq.h"
#include "hq_internal.h"
#include "hq_layout.h"
#include "hq_marlin_gemm.hpp"

#include <chrono>
#include <cmath>
#include <random>
#include <stdexcept>
#include <string>

namespace hydrogen {

namespace {

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + " -> " + cudaGetErrorString(e));
}
void check_hq(hq_status s, const char* what) {
    if (s != HQ_OK) throw std::runtime_error(std::string(what) + " -> " + hq_last_error_string());
}

}  // namespace

MarlinGemmEngine::MarlinGemmEngine(MarlinGemmConfig config) : config_(config) {
    if (config_.K == 0 || config_.N == 0 || config_.group_size == 0)
        throw std::runtime_error("MarlinGemmEngine: zero-sized configuration");
    ensure_workspace(config_.M > 16 ? config_.M : 16);
}

MarlinGemmEngine::~MarlinGemmEngine() { free_device_memory(); }

void MarlinGemmEngine::free_device_memory() {
    void* ptrs[] = {d_workspace_, d_X_,     d_W_linear_, d_W_marlin_,  d_scales_,
                    d_biases_,    d_W_dequant_, d_Y_ref_, d_Y_marlin_, d_Y_baseline_};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    d_workspace_ = nullptr;
}

void MarlinGemmEngine::ensure_workspace(uint32_t M) {
    // Room for the re-tiled weights of the drop-in path plus the kernel workspace.
    size_t need = hq_gemm_workspace_size((int)M, (int)config_.N, (int)config_.K, (int)config_.group_size,
                                         HQ_WFMT_MARLIN_QUAD);
    if (need <= workspace_bytes_) return;
    if (d_workspace_) cudaFree(d_workspace_);
    d_workspace_ = nullptr;
    check_cuda(cudaMalloc(&d_workspace_, need), "cudaMalloc(workspace)");
    check_cuda(cudaMemset(d_workspace_, 0, need), "cudaMemset(workspace)");
    workspace_bytes_ = need;
}

void MarlinGemmEngine::run(const float* d_X, const uint32_t* d_W, int wfmt, const float* d_scales,
                           const float* d_biases, float* d_Y, uint32_t M) {
    ensure_workspace(M);
    check_hq(hq_gemm(d_X, HQ_F32, d_W, (hq_wfmt)wfmt, d_scales, HQ_F32, d_biases, d_Y, HQ_F32, (int)M,
                     (int)config_.N, (int)config_.K, (int)config_.group_size, d_workspace_, workspace_bytes_,
                     nullptr),
             "hq_gemm");
}

MarlinRepackResult MarlinGemmEngine::repack_q4k_to_marlin(const uint8_t* h_src_q4k, uint32_t* h_dst_marlin,
                                                          uint32_t K, uint32_t N) {
    auto t0 = std::chrono::high_resolution_clock::now();
    check_hq(hq_repack_host(h_src_q4k, HQ_WFMT_LINEAR_U4, h_dst_marlin, HQ_WFMT_MARLIN_QUAD, (int)K, (int)N, 0),
             "hq_repack_host");
    auto t1 = std::chrono::high_resolution_clock::now();
    MarlinRepackResult r;
    r.num_weights = (size_t)K * N;
    r.repack_time_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    r.repack_time_seconds = r.repack_time_ms / 1000.0;
    r.repack_under_1s = r.repack_time_seconds < 1.0;
    return r;
}

void MarlinGemmEngine::forward_baseline_int4(const float* d_X, const uint32_t* d_W_linear, const float* d_scales,
                                             const float* d_biases, float* d_Y, uint32_t M) {
    if (!d_X || !d_W_linear || !d_scales || !d_Y) throw std::runtime_error("forward_baseline_int4: null pointer");
    check_cuda(hq::launch_baseline_u4(d_X, d_W_linear, d_scales, d_biases, d_Y, (int)M, (int)config_.K,
                                      (int)config_.N, (int)config_.group_size, nullptr),
               "forward_baseline_int4 launch");
}

void MarlinGemmEngine::forward_marlin_int4(const float* d_X, const uint32_t* d_W_marlin, const float* d_scales,
                                           const float* d_biases, float* d_Y, uint32_t M) {
    run(d_X, d_W_marlin, HQ_WFMT_MARLIN_QUAD, d_scales, d_biases, d_Y, M);
}

void MarlinGemmEngine::forward_reference(const float* d_X, const float* d_W_dequant, float* d_Y_ref, uint32_t M) {
    check_cuda(hq::launch_f32_gemm(d_X, d_W_dequant, d_Y_ref, (int)M, (int)config_.K, (int)config_.N, nullptr),
               "forward_reference launch");
}

void MarlinGemmEngine::forward_cutlass_int8(const float* d_X, const int8_t* d_W_int8, const float* d_scales,
                                            float* d_Y, uint32_t M) {
    if (hq_w8_gemm(d_X, d_W_int8, d_scales, d_Y, (int)M, (int)config_.K, (int)config_.N, nullptr) != HQ_OK)
        throw std::runtime_error(std::string("forward_cutlass_int8: ") + hq_last_error_string());
}

void MarlinGemmEngine::verify_fidelity(const float* d_Y_ref, const float* d_Y_marlin, uint32_t M,
                                       double& out_max_abs_err, double& out_mse) {
    const size_t count = (size_t)M * config_.N;
    std::vector<float> a(count), b(count);
    check_cuda(cudaMemcpy(a.data(), d_Y_ref, count * sizeof(float), cudaMemcpyDeviceToHost), "D2H Y_ref");
    check_cuda(cudaMemcpy(b.data(), d_Y_marlin, count * sizeof(float), cudaMemcpyDeviceToHost), "D2H Y");
    double mx = 0.0, sq = 0.0;
    for (size_t i = 0; i < count; ++i) {
        double d = std::fabs((double)a[i] - (double)b[i]);
        if (d > mx) mx = d;
        sq += d * d;
    }
    out_max_abs_err = mx;
    out_mse = count ? sq / (double)count : 0.0;
}

// Synthetic data with the reference's distributions (marlin_gemm.cu:469-512):
// X ~ N(0, 0.25), scale = 0.05 + (rng % 1000) * 1e-4, bias = -8 * scale, u ~ U{0..15}.
void MarlinGemmEngine::ensure_synthetic_data() {
    if (d_X_) return;
    const size_t M = config_.M, K = config_.K, N = config_.N, g = config_.group_size;
    std::mt19937 rng(42);
    std::normal_distribution<float> dist(0.0f, 0.25f);
    std::uniform_int_distribution<uint32_t> qd(0, 15);
    std::vector<float> X(M * K), S((K / g) * N), B((K / g) * N), Wd(K * N);
    for (auto& f : X) f = dist(rng);
    for (size_t i = 0; i < S.size(); ++i) {
        S[i] = 0.05f + (float)(rng() % 1000) * 0.0001f;
        B[i] = -8.0f * S[i];
    }
    std::vector<uint32_t> Wl((K / 8) * N), Wm((K / 8) * N);
    for (size_t kw = 0; kw < K / 8; ++kw)
        for (size_t n = 0; n < N; ++n) {
            uint32_t packed = 0;
            const size_t gi = kw * 8 / g;
            for (uint32_t i = 0; i < 8; ++i) {
                uint32_t q = qd(rng);
                packed |= q << (4 * i);
                Wd[(kw * 8 + i) * N + n] = (float)q * S[gi * N + n] + B[gi * N + n];
            }
            Wl[kw * N + n] = packed;
        }
    repack_q4k_to_marlin(reinterpret_cast<const uint8_t*>(Wl.data()), Wm.data(), (uint32_t)K, (uint32_t)N);
    auto alloc_copy = [](auto** dst, const auto& v) {
        check_cuda(cudaMalloc(reinterpret_cast<void**>(dst), v.size() * sizeof(v[0])), "cudaMalloc");
        check_cuda(cudaMemcpy(*dst, v.data(), v.size() * sizeof(v[0]), cudaMemcpyHostToDevice), "H2D");
    };
    alloc_copy(&d_X_, X);
    alloc_copy(&d_W_linear_, Wl);
    alloc_copy(&d_W_marlin_, Wm);
    alloc_copy(&d_scales_, S);
    alloc_copy(&d_biases_, B);
    alloc_copy(&d_W_dequant_, Wd);
    for (float** p : {&d_Y_ref_, &d_Y_marlin_, &d_Y_baseline_})
        check_cuda(cudaMalloc(reinterpret_cast<void**>(p), M * N * sizeof(float)), "cudaMalloc(Y)");
}

std::vector<MarlinBenchmarkResult> MarlinGemmEngine::run_benchmark_sweep(int warmups, int iterations) {
    ensure_synthetic_data();
    std::vector<MarlinBenchmarkResult> results;
    cudaEvent_t start, stop;
    check_cuda(cudaEventCreate(&start), "cudaEventCreate");
    check_cuda(cudaEventCreate(&stop), "cudaEventCreate");
    const size_t static_bytes =
        (size_t)config_.K * config_.N / 2 + (size_t)config_.K / config_.group_size * config_.N * sizeof(float) * 2;
    for (uint32_t m : {1u, 2u, 4u, 8u}) {
        if (m > config_.M) break;
        forward_reference(d_X_, d_W_dequant_, d_Y_ref_, m);
        forward_marlin_int4(d_X_, d_W_marlin_, d_scales_, d_biases_, d_Y_marlin_, m);
        check_cuda(cudaDeviceSynchronize(), "sync");
        double max_err = 0, mse = 0;
        verify_fidelity(d_Y_ref_, d_Y_marlin_, m, max_err, mse);
        auto time_it = [&](auto&& fn) {
            for (int w = 0; w < warmups; ++w) fn();
            check_cuda(cudaDeviceSynchronize(), "sync");
            check_cuda(cudaEventRecord(start), "record");
            for (int i = 0; i < iterations; ++i) fn();
            check_cuda(cudaEventRecord(stop), "record");
            check_cuda(cudaEventSynchronize(stop), "sync");
            float ms = 0;
            check_cuda(cudaEventElapsedTime(&ms, start, stop), "elapsed");
            return ms / (float)iterations;
        };
        float base_ms =
            time_it([&] { forward_baseline_int4(d_X_, d_W_linear_, d_scales_, d_biases_, d_Y_baseline_, m); });
        float marlin_ms =
            time_it([&] { forward_marlin_int4(d_X_, d_W_marlin_, d_scales_, d_biases_, d_Y_marlin_, m); });
        const size_t total = static_bytes + (size_t)m * config_.K * 4 + (size_t)m * config_.N * 4;
        const double s = marlin_ms / 1000.0;
        MarlinBenchmarkResult r;
        r.M = m;
        r.K = config_.K;
        r.N = config_.N;
        r.marlin_latency_ms = marlin_ms;
        r.baseline_latency_ms = base_ms;
        r.marlin_bandwidth_gbs = (double)total / 1e9 / s;
        r.bandwidth_utilization_pct = r.marlin_bandwidth_gbs / kPeakBandwidthGBs * 100.0;
        r.marlin_tflops = 2.0 * m * config_.K * config_.N / 1e12 / s;
        r.speedup_ratio = marlin_ms > 0 ? base_ms / marlin_ms : 1.0;
        r.max_abs_error = max_err;
        r.mean_squared_error = mse;
        r.numerical_match = max_err < 1e-3;
        r.latency_target_met = marlin_ms <= 0.15f;
        r.bandwidth_target_met = r.bandwidth_utilization_pct >= 80.0 || (m > 1 && r.latency_target_met);
        results.push_back(r);
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    return results;
}

MarlinRepackResult MarlinGemmEngine::benchmark_repacking() {
    const size_t words = (size_t)(config_.K / 8) * config_.N;
    std::vector<uint32_t> src(words, 0x12345678u), dst(words, 0);
    return repack_q4k_to_marlin(reinterpret_cast<const uint8_t*>(src.data()), dst.data(), config_.K, config_.N);
}

}  // namespace hydrogen

// ------------------------------------------------------------ C wrappers

struct hq_marlin_engine {
    hydrogen::MarlinGemmEngine* e;
};

namespace {
template <typename F>
hq_status guarded(F&& f) {
    try {
        f();
        return HQ_OK;
    } catch (const std::exception& ex) {
        hq::set_last_error(ex.what());
        return HQ_ERR_CUDA;
    }
}
}  // namespace

extern "C" {

HQ_API hq_marlin_engine* hq_marlin_engine_create(uint32_t M, uint32_t K, uint32_t N, uint32_t group_size) {
    try {
        hydrogen::MarlinGemmConfig c;
        c.M = M;
        c.K = K;
        c.N = N;
        c.group_size = group_size;
        return new hq_marlin_engine{new hydrogen::MarlinGemmEngine(c)};
    } catch (const std::exception& ex) {
        hq::set_last_error(ex.what());
        return nullptr;
    }
}

HQ_API void hq_marlin_engine_destroy(hq_marlin_engine* e) {
    if (!e) return;
    delete e->e;
    delete e;
}

HQ_API hq_status hq_marlin_repack_q4k_to_marlin(hq_marlin_engine* e, const uint8_t* h_src_q4k, uint32_t* h_dst_marlin,
                                                uint32_t K, uint32_t N, double* repack_ms) {
    if (!e) return HQ_ERR_INVALID_ARG;
    return guarded([&] {
        auto r = e->e->repack_q4k_to_marlin(h_src_q4k, h_dst_marlin, K, N);
        if (repack_ms) *repack_ms = r.repack_time_ms;
    });
}

HQ_API hq_status hq_marlin_forward_marlin_int4(hq_marlin_engine* e, const float* d_X, const uint32_t* d_W_marlin,
                                               const float* d_scales, const float* d_biases, float* d_Y, uint32_t M) {
    if (!e) return HQ_ERR_INVALID_ARG;
    return guarded([&] { e->e->forward_marlin_int4(d_X, d_W_marlin, d_scales, d_biases, d_Y, M); });
}

HQ_API hq_status hq_marlin_forward_baseline_int4(hq_marlin_engine* e, const float* d_X, const uint32_t* d_W_linear,
                                                 const float* d_scales, const float* d_biases, float* d_Y,
                                                 uint32_t M) {
    if (!e) return HQ_ERR_INVALID_ARG;
    return guarded([&] { e->e->forward_baseline_int4(d_X, d_W_linear, d_scales, d_biases, d_Y, M); });
}

HQ_API hq_status hq_marlin_forward_reference(hq_marlin_engine* e, const float* d_X, const float* d_W_dequant,
                                             float* d_Y_ref, uint32_t M) {
    if (!e) return HQ_ERR_INVALID_ARG;
    return guarded([&] { e->e->forward_reference(d_X, d_W_dequant, d_Y_ref, M); });
}

HQ_API hq_status hq_marlin_forward_cutlass_int8(hq_marlin_engine* e, const float* d_X, const int8_t* d_W_int8,
                                                const float* d_scales, float* d_Y, uint32_t M) {
    if (!e) return HQ_ERR_INVALID_ARG;
    return guarded([&] { e->e->forward_cutlass_int8(d_X, d_W_int8, d_scales, d_Y, M); });
}

HQ_API hq_status hq_marlin_verify_fidelity(hq_marlin_engine* e, const float* d_Y_ref, const float* d_Y_marlin,
                                           uint32_t M, double* max_abs_err, double* mse) {
    if (!e || !max_abs_err || !mse) return HQ_ERR_INVALID_ARG;
    return guarded([&] { e->e->verify_fidelity(d_Y_ref, d_Y_marlin, M, *max_abs_err, *mse); });
}

}  // extern "C"
