// hq_noalloc.cu -- hq_gemm for callers that cannot allocate device memory.
//
// hq_gemm takes a caller-owned workspace: reference-layout weights
// (LINEAR_U4, MARLIN_QUAD, LINEAR_T2) are re-tiled into it before the GEMM
// reads them.  Some hosts cannot provide one: a plugin loaded into a serving
// process whose device memory is owned and budgeted by that process (a
// pre-sized arena, another framework's caching allocator) may not call
// cudaMalloc at all, and a cudaMalloc in the middle of a step would also
// synchronise the device.  hq_gemm_noalloc gives them the same operation
// with the workspace in a fixed array compiled into this library instead.
//
// The array is a file-scope __device__ variable of HQ_NOALLOC_SCRATCH_BYTES.
// Host code only sees a stand-in symbol for it, so the device address is
// looked up with cudaGetSymbolAddress, once per device, on the first call
// made with that device current.  That first call also zero-fills the array
// (hq_gemm's workspace contract: the decode kernel keeps per-column-group
// arrival counters there, zero before first use and left at zero by every
// call) and waits for the fill to finish with cudaDeviceSynchronize, so that
// no kernel of this or any later call, on any stream, can overtake it.  The
// first call on a device must therefore come before any stream capture.
// The array belongs to the library's device code: it is resident on every
// device where the library's module is loaded (at the first call under lazy
// module loading, at context creation with CUDA_MODULE_LOADING=EAGER) until
// the process exits.
//
// Every call on a device shares the one array and finds there whatever the
// previous call left.  Calls whose GPU work overlaps (concurrent streams,
// several host threads) race on it; serialise them on one stream.
#include "hq.h"
#include "hq_internal.h"

#include <cstdio>
#include <mutex>

namespace hq {
namespace {

constexpr size_t kScratchBytes = HQ_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

hq_status noalloc_fail(hq_status s, const char* msg) {
    set_last_error(msg);
    return s;
}

// Device address of the array on the current device (set-up on first use).
hq_status scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return noalloc_fail(HQ_ERR_CUDA, "hq_gemm_noalloc: cudaGetDevice failed");
    if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(HQ_ERR_INVALID_ARG, "hq_gemm_noalloc: device ordinal >= 64");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            char buf[160];
            snprintf(buf, sizeof buf, "hq_gemm_noalloc: cudaGetSymbolAddress(scratch) failed: %s",
                     cudaGetErrorString(e));
            return noalloc_fail(HQ_ERR_CUDA, buf);
        }
        e = cudaMemset(p, 0, kScratchBytes);
        // cudaMemset on device memory may return before the fill is done, and
        // it is not ordered with the caller's (possibly non-blocking) stream.
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            char buf[160];
            snprintf(buf, sizeof buf, "hq_gemm_noalloc: zero-filling the scratch array failed: %s",
                     cudaGetErrorString(e));
            return noalloc_fail(HQ_ERR_CUDA, buf);
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return HQ_OK;
}

}  // namespace
}  // namespace hq

extern "C" HQ_API hq_status hq_gemm_noalloc(const void* A, hq_dtype a_dtype, const void* Wq, hq_wfmt wfmt,
                                            const void* scales, hq_dtype s_dtype, const float* bias, void* C,
                                            hq_dtype c_dtype, int M, int N, int K, int group,
                                            hq_stream_t stream) {
    // Bad shapes and formats get hq_gemm's own diagnostics (workspace size 0 here).
    const size_t need = hq_gemm_workspace_size(M, N, K, group, wfmt);
    if (need == 0)  // nothing to hold: no set-up, no scratch
        return hq_gemm(A, a_dtype, Wq, wfmt, scales, s_dtype, bias, C, c_dtype, M, N, K, group, nullptr, 0, stream);
    if (need > hq::kScratchBytes) {
        char buf[200];
        snprintf(buf, sizeof buf,
                 "hq_gemm_noalloc: this problem needs %zu bytes of scratch (M=%d N=%d K=%d), more than the "
                 "%zu-byte static array; use hq_gemm with a caller workspace or tile-order weights",
                 need, M, N, K, (size_t)hq::kScratchBytes);
        return hq::noalloc_fail(HQ_ERR_WORKSPACE_TOO_SMALL, buf);
    }
    void* scratch = nullptr;
    const hq_status st = hq::scratch_address(&scratch);
    if (st != HQ_OK) return st;
    return hq_gemm(A, a_dtype, Wq, wfmt, scales, s_dtype, bias, C, c_dtype, M, N, K, group, scratch,
                   hq::kScratchBytes, stream);
}
