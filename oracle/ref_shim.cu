// ref_shim.cu -- C entry points into the reference's own MarlinGemmEngine.
//
// TEST INFRASTRUCTURE ONLY.  Linked with the reference's unmodified
// hydrogen/src/model/marlin_gemm.cu (compiled where it lies) into
// oracle/_ref/libref_marlin.so so that tests can run the reference's host
// repack, its kernel_reference_gemm and its Marlin kernel on a B200 against
// this project's oracle.  Every entry point works on a constructed engine.  Exceptions thrown by
// the reference (CUDA_CHECK, marlin_gemm.cu:19-27) become return code -1.
#include "marlin_gemm.hpp"

#include <cstdint>
#include <cstring>
#include <exception>

namespace {
char g_err[512];
void set_err(const char* s) {
    std::strncpy(g_err, s, sizeof g_err - 1);
    g_err[sizeof g_err - 1] = 0;
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err; }

// MarlinGemmEngine::repack_q4k_to_marlin (marlin_gemm.cu:432-467) called on a
// constructed engine (ref_engine_create).  The constructor allocates device
// memory (:381-385, :391-416), so this needs a GPU.
int ref_engine_repack_q4k_to_marlin(void* e, const uint32_t* src, uint32_t* dst, uint32_t K, uint32_t N,
                                    double* ms_out) {
    try {
        hydrogen::MarlinRepackResult r = static_cast<hydrogen::MarlinGemmEngine*>(e)->repack_q4k_to_marlin(
            reinterpret_cast<const uint8_t*>(src), dst, K, N);
        if (ms_out) *ms_out = r.repack_time_ms;
        return 0;
    } catch (const std::exception& ex) {
        set_err(ex.what());
        return -1;
    }
}

void* ref_engine_create(uint32_t M, uint32_t K, uint32_t N, uint32_t group) {
    try {
        hydrogen::MarlinGemmConfig c;
        c.M = M;
        c.K = K;
        c.N = N;
        c.group_size = group;
        return new hydrogen::MarlinGemmEngine(c);
    } catch (const std::exception& e) {
        set_err(e.what());
        return nullptr;
    }
}

void ref_engine_destroy(void* e) { delete static_cast<hydrogen::MarlinGemmEngine*>(e); }

int ref_forward_reference(void* e, const float* dX, const float* dW, float* dY, uint32_t M) {
    try {
        static_cast<hydrogen::MarlinGemmEngine*>(e)->forward_reference(dX, dW, dY, M);
        return 0;
    } catch (const std::exception& ex) {
        set_err(ex.what());
        return -1;
    }
}

int ref_forward_marlin(void* e, const float* dX, const uint32_t* dWq, const float* ds,
                       const float* db, float* dY, uint32_t M) {
    try {
        static_cast<hydrogen::MarlinGemmEngine*>(e)->forward_marlin_int4(dX, dWq, ds, db, dY, M);
        return 0;
    } catch (const std::exception& ex) {
        set_err(ex.what());
        return -1;
    }
}

int ref_forward_baseline(void* e, const float* dX, const uint32_t* dWl, const float* ds,
                         const float* db, float* dY, uint32_t M) {
    try {
        static_cast<hydrogen::MarlinGemmEngine*>(e)->forward_baseline_int4(dX, dWl, ds, db, dY, M);
        return 0;
    } catch (const std::exception& ex) {
        set_err(ex.what());
        return -1;
    }
}

int ref_forward_cutlass_int8(void* e, const float* dX, const int8_t* dW, const float* ds, float* dY, uint32_t M) {
    try {
        static_cast<hydrogen::MarlinGemmEngine*>(e)->forward_cutlass_int8(dX, dW, ds, dY, M);
        return 0;
    } catch (const std::exception& ex) {
        set_err(ex.what());
        return -1;
    }
}

}  // extern "C"
