// hq_api.cu -- the C ABI (include/hq.h): argument checking, dispatch, errors.
//
// Nothing here throws across the ABI and nothing allocates: every device
// buffer is the caller's, including the workspace.
#include "hq.h"
#include "hq_common.cuh"
#include "hq_internal.h"
#include "hq_layout.h"

#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <string>
#include <utility>
#include <vector>

namespace hq {

// The one device error word of the library (see hq_common.cuh).
__device__ unsigned g_dev_error_word = 0;

const DeviceInfo& device_info(int dev) {
    static std::mutex mu;
    static std::vector<DeviceInfo> cache(128);
    static std::vector<bool> have(128, false);
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 128) dev = 0;
    if (!have[dev]) {
        DeviceInfo d{};
        cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        d.smem_optin = (size_t)optin;
        if (d.sm_count <= 0) d.sm_count = 148;
        cache[dev] = d;
        have[dev] = true;
    }
    return cache[dev];
}

// The attribute is a per-kernel maximum: keep the largest size set on each device and only
// ever raise it, so that a launch with less shared memory never lowers it under another.
cudaError_t ensure_smem_attr(const void* fn, int dev, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> set_max;
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_pair(fn, dev);
    auto it = set_max.find(key);
    if (it != set_max.end() && it->second >= bytes) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) set_max[key] = bytes;
    return e;
}

int max_active_clusters(const void* fn, int threads, int smem, int cs, int dev) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, int, int>, int> cache;
    std::lock_guard<std::mutex> lk(mu);
    const auto key = std::make_tuple(fn, threads, smem, cs, dev);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    if (cs > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        (void)cudaGetLastError();
        return cache[key] = 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(cs * 64));
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int v = 0;
    if (cudaOccupancyMaxActiveClusters(&v, fn, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        v = 0;
    }
    return cache[key] = v;
}

unsigned* device_error_word(int dev) {
    static std::mutex mu;
    static std::vector<unsigned*> cache(128, nullptr);
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 128) return nullptr;
    if (!cache[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_error_word) == cudaSuccess) cache[dev] = static_cast<unsigned*>(p);
    }
    return cache[dev];
}

cudaError_t read_and_clear_device_error(unsigned* code) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return e;
    unsigned v = 0;
    e = cudaMemcpyFromSymbol(&v, g_dev_error_word, sizeof v);
    if (e != cudaSuccess) return e;
    if (v) {
        unsigned z = 0;
        e = cudaMemcpyToSymbol(g_dev_error_word, &z, sizeof z);
    }
    *code = v;
    return e;
}

}  // namespace hq

using namespace hq;

namespace {
thread_local std::string t_last_error;
}  // namespace

void hq::set_last_error(const char* msg) { t_last_error = msg ? msg : ""; }

namespace {

hq_status fail(hq_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return s;
}

hq_status cuda_fail(cudaError_t e, const char* what) {
    return fail(HQ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

bool valid_dtype(int d) { return d == HQ_F32 || d == HQ_F16 || d == HQ_BF16; }

int fmt_wbits(hq_wfmt f) {
    switch (f) {
        case HQ_WFMT_LINEAR_U4:
        case HQ_WFMT_MARLIN_QUAD:
        case HQ_WFMT_TILE_U4:
        case HQ_WFMT_TILE_U4_K32: return 4;
        case HQ_WFMT_LINEAR_T2:
        case HQ_WFMT_TILE_T2: return 2;
        default: return 0;
    }
}
bool fmt_is_tile(hq_wfmt f) { return f == HQ_WFMT_TILE_U4 || f == HQ_WFMT_TILE_T2 || f == HQ_WFMT_TILE_U4_K32; }

hq_status check_shape(int M, int N, int K, int group) {
    if (M < 0 || N <= 0 || K <= 0) return fail(HQ_ERR_INVALID_ARG, "negative or zero size M=%d N=%d K=%d", M, N, K);
    if (N % 16) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "N=%d must be a multiple of 16", N);
    if (K % 64) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "K=%d must be a multiple of 64", K);
    if (group <= 0 || (group % 64 && group != 32) || K % group)
        return fail(HQ_ERR_UNSUPPORTED_SHAPE, "group=%d must be 32 or a multiple of 64 dividing K=%d", group, K);
    return HQ_OK;
}

hq_status check_device(int* dev_out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    const DeviceInfo& di = device_info(dev);
    if (di.cc_major != 10) return fail(HQ_ERR_UNSUPPORTED_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                                       dev, di.cc_major, di.cc_minor);
    *dev_out = dev;
    return HQ_OK;
}

size_t kernel_ws(int M, int N, int K, int wbits, int dev) {
    const int Md = M <= 16 ? M : 16;
    size_t d = M > 0 ? decode_workspace_bytes(Md, N, K, wbits, dev) : 0;
    size_t p = M > 16 ? prefill_workspace_bytes(M, N, K, wbits, dev) : 0;
    return up256(d > p ? d : p);
}

}  // namespace

extern "C" {

HQ_API const char* hq_version(void) { return "hq 0.1.0 sm_100a"; }

HQ_API const char* hq_last_error_string(void) { return t_last_error.c_str(); }

HQ_API size_t hq_weight_bytes(hq_wfmt fmt, int K, int N) {
    if (K <= 0 || N <= 0) return 0;
    switch (fmt) {
        case HQ_WFMT_LINEAR_U4:
        case HQ_WFMT_MARLIN_QUAD: return (K % 8 || (fmt == HQ_WFMT_MARLIN_QUAD && K % 32)) ? 0 : (size_t)K * N / 2;
        case HQ_WFMT_LINEAR_T2: return K % 16 ? 0 : (size_t)K * N / 4;
        case HQ_WFMT_TILE_U4:
        case HQ_WFMT_TILE_U4_K32:
        case HQ_WFMT_TILE_T2:
            if (K % 64 || N % 16) return 0;
            return TileGeom(K, N, fmt_wbits(fmt)).bytes();
        case HQ_WFMT_TQ1_0: return K % 256 ? 0 : (size_t)N * (K / 256) * 56;
    }
    return 0;
}

HQ_API size_t hq_gemm_workspace_size(int M, int N, int K, int group, hq_wfmt wfmt) {
    const int wbits = fmt_wbits(wfmt);
    if (!wbits || M < 0 || N <= 0 || K <= 0 || N % 16 || K % 64 || group <= 0 || K % group) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    size_t retile = fmt_is_tile(wfmt) ? 0 : up256(TileGeom(K, N, wbits).bytes());
    return retile + kernel_ws(M, N, K, wbits, dev);
}

HQ_API hq_status hq_workspace_init(void* workspace, size_t ws_bytes, hq_stream_t stream) {
    if (!workspace && ws_bytes) return fail(HQ_ERR_INVALID_ARG, "null workspace");
    if (!ws_bytes) return HQ_OK;
    cudaError_t e = cudaMemsetAsync(workspace, 0, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "cudaMemsetAsync(workspace)");
}

HQ_API hq_status hq_gemm(const void* A, hq_dtype a_dtype, const void* Wq, hq_wfmt wfmt, const void* scales,
                         hq_dtype s_dtype, const float* bias, void* C, hq_dtype c_dtype, int M, int N, int K,
                         int group, void* workspace, size_t ws_bytes, hq_stream_t stream) {
    hq_status st = check_shape(M, N, K, group);
    if (st != HQ_OK) return st;
    if (M == 0) return HQ_OK;
    const int wbits = fmt_wbits(wfmt);
    if (!wbits) return fail(HQ_ERR_INVALID_ARG, "unsupported weight format %d for hq_gemm", (int)wfmt);
    if (!valid_dtype(a_dtype) || !valid_dtype(s_dtype) || !valid_dtype(c_dtype))
        return fail(HQ_ERR_INVALID_ARG, "bad dtype enum");
    if (!A || !Wq || !scales || !C) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (!aligned16(A) || !aligned16(Wq) || !aligned16(C) || !aligned16(workspace) || !aligned16(scales) ||
        (bias && !aligned16(bias)))
        return fail(HQ_ERR_MISALIGNED, "A, Wq, scales, bias, C and workspace must be 16-byte aligned");
    if (bias && wbits != 4) return fail(HQ_ERR_INVALID_ARG, "bias is only defined for int4 weights");
    if (wfmt == HQ_WFMT_TILE_U4_K32 && group != 32)
        return fail(HQ_ERR_INVALID_ARG, "HQ_WFMT_TILE_U4_K32 is the group-32 layout (group=%d)", group);
    if (group == 32 && (wfmt == HQ_WFMT_TILE_U4 || wbits != 4))
        return fail(HQ_ERR_INVALID_ARG, "group 32 takes int4 weights in HQ_WFMT_TILE_U4_K32 (hq_repack_*, "
                                        "hq_q4_k_to_tile) or a reference layout");
    int dev = 0;
    if ((st = check_device(&dev)) != HQ_OK) return st;

    const size_t need = hq_gemm_workspace_size(M, N, K, group, wfmt);
    if (need && !workspace) return fail(HQ_ERR_INVALID_ARG, "null workspace (%zu bytes required)", need);
    if (ws_bytes < need) return fail(HQ_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < required %zu", ws_bytes, need);

    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const uint8_t* W = static_cast<const uint8_t*>(Wq);
    if (!fmt_is_tile(wfmt)) {
        // Drop-in path: re-tile the reference layout into the workspace first.
        uint8_t* tile = ws;
        cudaError_t e = launch_linear_to_tile(Wq, wfmt == HQ_WFMT_MARLIN_QUAD, wbits, tile, K, N, s, group == 32);
        if (e != cudaSuccess) return cuda_fail(e, "re-tile launch");
        W = tile;
        ws += up256(TileGeom(K, N, wbits).bytes());
    }

    GemmArgs a;
    a.A = A;
    a.a_dtype = (DType)a_dtype;
    a.W = W;
    a.wbits = wbits;
    a.S = scales;
    a.s_dtype = (DType)s_dtype;
    a.bias = bias;
    a.C = C;
    a.c_dtype = (DType)c_dtype;
    a.N = N;
    a.K = K;
    a.group = group;
    a.weights_just_written = !fmt_is_tile(wfmt);
    a.ws = ws;
    a.ws_bytes = workspace ? ws_bytes - (size_t)(ws - static_cast<uint8_t*>(workspace)) : 0;
    a.stream = s;

    if (M > 16) {
        a.M = M;
        if (prefill_supported(a)) {
            cudaError_t e = launch_prefill(a);
            return e == cudaSuccess ? HQ_OK : cuda_fail(e, "tensor-core kernel launch");
        }
    }
    // Decode kernel, 16 rows at a time.
    a.M = M < 16 ? M : 16;
    if (!decode_supported(a))
        return fail(HQ_ERR_INVALID_ARG, "unsupported dtype combination a=%d s=%d c=%d bias=%d wbits=%d", (int)a_dtype,
                    (int)s_dtype, (int)c_dtype, bias != nullptr, wbits);
    const size_t a_row = (size_t)K * (a_dtype == HQ_F32 ? 4 : 2);
    const size_t c_row = (size_t)N * (c_dtype == HQ_F32 ? 4 : 2);
    for (int m0 = 0; m0 < M; m0 += 16) {
        a.M = M - m0 < 16 ? M - m0 : 16;
        a.A = static_cast<const uint8_t*>(A) + (size_t)m0 * a_row;
        a.C = static_cast<uint8_t*>(C) + (size_t)m0 * c_row;
        cudaError_t e = launch_decode(a);
        if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
    }
    return HQ_OK;
}

HQ_API hq_status hq_repack_host(const void* src, hq_wfmt src_fmt, void* dst, hq_wfmt dst_fmt, int K, int N,
                                int nthreads) {
    if (!src || !dst) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (K <= 0 || N <= 0) return fail(HQ_ERR_INVALID_ARG, "bad size");
    const uint32_t* s = static_cast<const uint32_t*>(src);
    uint32_t* d = static_cast<uint32_t*>(dst);
    if (src_fmt == HQ_WFMT_LINEAR_U4 && dst_fmt == HQ_WFMT_MARLIN_QUAD) {
        if (K % 32) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "K %% 32 != 0");
        host::linear_quad(s, d, K, N, false, nthreads);
        return HQ_OK;
    }
    if (src_fmt == HQ_WFMT_MARLIN_QUAD && dst_fmt == HQ_WFMT_LINEAR_U4) {
        if (K % 32) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "K %% 32 != 0");
        host::linear_quad(s, d, K, N, true, nthreads);
        return HQ_OK;
    }
    if (K % 64 || N % 16) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "tile order needs K %% 64 == 0 and N %% 16 == 0");
    const bool k32 = dst_fmt == HQ_WFMT_TILE_U4_K32 || src_fmt == HQ_WFMT_TILE_U4_K32;
    if ((src_fmt == HQ_WFMT_LINEAR_U4 || src_fmt == HQ_WFMT_MARLIN_QUAD) &&
        (dst_fmt == HQ_WFMT_TILE_U4 || dst_fmt == HQ_WFMT_TILE_U4_K32)) {
        host::linear_to_tile(s, src_fmt == HQ_WFMT_MARLIN_QUAD, 4, d, K, N, nthreads, k32);
        return HQ_OK;
    }
    if ((src_fmt == HQ_WFMT_TILE_U4 || src_fmt == HQ_WFMT_TILE_U4_K32) && dst_fmt == HQ_WFMT_LINEAR_U4) {
        host::tile_to_linear(s, 4, d, K, N, nthreads, k32);
        return HQ_OK;
    }
    if (src_fmt == HQ_WFMT_LINEAR_T2 && dst_fmt == HQ_WFMT_TILE_T2) {
        host::linear_to_tile(s, false, 2, d, K, N, nthreads);
        return HQ_OK;
    }
    if (src_fmt == HQ_WFMT_TILE_T2 && dst_fmt == HQ_WFMT_LINEAR_T2) {
        host::tile_to_linear(s, 2, d, K, N, nthreads);
        return HQ_OK;
    }
    return fail(HQ_ERR_INVALID_ARG, "unsupported repack %d -> %d", (int)src_fmt, (int)dst_fmt);
}

HQ_API hq_status hq_repack_device(const void* src, hq_wfmt src_fmt, void* dst, hq_wfmt dst_fmt, int K, int N,
                                  hq_stream_t stream) {
    if (!src || !dst) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (K <= 0 || N <= 0) return fail(HQ_ERR_INVALID_ARG, "bad size");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const uint32_t* sp = static_cast<const uint32_t*>(src);
    uint32_t* dp = static_cast<uint32_t*>(dst);
    cudaError_t e = cudaSuccess;
    if (src_fmt == HQ_WFMT_LINEAR_U4 && dst_fmt == HQ_WFMT_MARLIN_QUAD) {
        if (K % 32) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "K %% 32 != 0");
        e = launch_linear_to_quad(sp, dp, K, N, false, s);
    } else if (src_fmt == HQ_WFMT_MARLIN_QUAD && dst_fmt == HQ_WFMT_LINEAR_U4) {
        if (K % 32) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "K %% 32 != 0");
        e = launch_linear_to_quad(sp, dp, K, N, true, s);
    } else {
        if (K % 64 || N % 16) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "tile order needs K %% 64 == 0 and N %% 16 == 0");
        const bool k32 = dst_fmt == HQ_WFMT_TILE_U4_K32 || src_fmt == HQ_WFMT_TILE_U4_K32;
        if ((src_fmt == HQ_WFMT_LINEAR_U4 || src_fmt == HQ_WFMT_MARLIN_QUAD) &&
            (dst_fmt == HQ_WFMT_TILE_U4 || dst_fmt == HQ_WFMT_TILE_U4_K32))
            e = launch_linear_to_tile(src, src_fmt == HQ_WFMT_MARLIN_QUAD, 4, static_cast<uint8_t*>(dst), K, N, s,
                                      k32);
        else if ((src_fmt == HQ_WFMT_TILE_U4 || src_fmt == HQ_WFMT_TILE_U4_K32) && dst_fmt == HQ_WFMT_LINEAR_U4)
            e = launch_tile_to_linear(static_cast<const uint8_t*>(src), 4, dp, K, N, s, k32);
        else if (src_fmt == HQ_WFMT_LINEAR_T2 && dst_fmt == HQ_WFMT_TILE_T2)
            e = launch_linear_to_tile(src, false, 2, static_cast<uint8_t*>(dst), K, N, s);
        else if (src_fmt == HQ_WFMT_TILE_T2 && dst_fmt == HQ_WFMT_LINEAR_T2)
            e = launch_tile_to_linear(static_cast<const uint8_t*>(src), 2, dp, K, N, s);
        else
            return fail(HQ_ERR_INVALID_ARG, "unsupported repack %d -> %d", (int)src_fmt, (int)dst_fmt);
    }
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "repack launch");
}

HQ_API hq_status hq_q4_k_to_tile(const void* w_q4k, void* tile_u4, float* scales, float* bias, int K, int N,
                                    hq_stream_t stream) {
    if (!w_q4k || !tile_u4 || !scales || !bias) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (K <= 0 || N <= 0 || K % 256 || N % 16) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "need K %% 256 == 0, N %% 16 == 0");
    if (((uintptr_t)w_q4k & 7u) || ((uintptr_t)tile_u4 & 3u) || ((uintptr_t)scales & 3u) || ((uintptr_t)bias & 3u))
        return fail(HQ_ERR_MISALIGNED, "w_q4k must be 8-byte aligned, tile_u4 / scales / bias 4-byte aligned");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    cudaError_t e = launch_q4k_to_tile(static_cast<const uint8_t*>(w_q4k), static_cast<uint8_t*>(tile_u4), scales,
                                       bias, K, N, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "Q4_K conversion launch");
}

HQ_API hq_status hq_q4_k_to_tile_host(const void* w_q4k, void* tile_u4, float* scales, float* bias, int K, int N,
                                         int nthreads) {
    if (!w_q4k || !tile_u4 || !scales || !bias) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (K <= 0 || N <= 0 || K % 256 || N % 16) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "need K %% 256 == 0, N %% 16 == 0");
    host::q4k_to_tile(static_cast<const uint8_t*>(w_q4k), static_cast<uint32_t*>(tile_u4), scales, bias, K, N,
                      nthreads);
    return HQ_OK;
}

HQ_API hq_status hq_tq1_0_gemv(const float* x, const void* w, float* out, int in_dim, int out_dim,
                               hq_stream_t stream) {
    if (!x || !w || !out) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (in_dim <= 0 || out_dim <= 0) return fail(HQ_ERR_INVALID_ARG, "bad size");
    if (in_dim % 256) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "in_dim %% 256 != 0");
    if (((uintptr_t)w & 7u) || ((uintptr_t)x & 3u)) return fail(HQ_ERR_MISALIGNED, "w must be 8-byte aligned");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    if ((size_t)in_dim * 4 + 2048 > device_info(dev).smem_optin)
        return fail(HQ_ERR_UNSUPPORTED_SHAPE, "in_dim %d too large for the shared-memory x stage", in_dim);
    cudaError_t e = launch_tq1_0_gemv(x, static_cast<const uint8_t*>(w), out, in_dim, out_dim,
                                      reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "tq1_0 gemv launch");
}

HQ_API hq_status hq_tq1_0_to_tile_t2(const void* w_tq1, void* tile_t2, void* scales_f16, int K, int N,
                                     hq_stream_t stream) {
    if (!w_tq1 || !tile_t2 || !scales_f16) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (K <= 0 || N <= 0 || K % 256 || N % 16) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "need K %% 256 == 0, N %% 16 == 0");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    cudaError_t e = launch_tq1_0_to_tile_t2(static_cast<const uint8_t*>(w_tq1), static_cast<uint8_t*>(tile_t2),
                                            static_cast<uint16_t*>(scales_f16), K, N,
                                            reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "tq1_0 conversion launch");
}

HQ_API hq_status hq_w8_gemm(const float* X, const int8_t* W, const float* scales, float* Y, int M, int K, int N,
                            hq_stream_t stream) {
    if (!X || !W || !scales || !Y) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (M < 0 || K <= 0 || N <= 0) return fail(HQ_ERR_INVALID_ARG, "bad size");
    if (N % 4 || K > 65536) return fail(HQ_ERR_UNSUPPORTED_SHAPE, "need N %% 4 == 0 and K <= 65536");
    if (((uintptr_t)W & 3u) || ((uintptr_t)X & 3u) || ((uintptr_t)Y & 3u) || ((uintptr_t)scales & 3u))
        return fail(HQ_ERR_MISALIGNED, "W, X, Y and scales must be 4-byte aligned");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    if (M == 0) return HQ_OK;
    cudaError_t e = launch_w8_gemm(X, W, scales, Y, M, K, N, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "w8 gemm launch");
}

HQ_API hq_status hq_output_projection(const float* x, const void* w, int w_type, float* logits,
                                      int embedding_dim, int vocab_size, hq_stream_t stream) {
    if (!x || !w || !logits) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (embedding_dim <= 0 || vocab_size <= 0) return fail(HQ_ERR_INVALID_ARG, "bad size");
    const bool tq1 = w_type == HQ_GGML_TQ1_0 || w_type == HQ_GGML_TQ1_0_ALT;
    if (w_type != HQ_GGML_F32 && w_type != HQ_GGML_BF16 && w_type != HQ_GGML_Q8_0 && !tq1)
        return fail(HQ_ERR_INVALID_ARG, "w_type %d is not F32 (0), Q8_0 (8), BF16 (30) or TQ1_0 (34, 143)", w_type);
    if (tq1) return hq_tq1_0_gemv(x, w, logits, embedding_dim, vocab_size, stream);
    if (w_type == HQ_GGML_Q8_0 && embedding_dim % 32)
        return fail(HQ_ERR_UNSUPPORTED_SHAPE, "Q8_0 needs embedding_dim %% 32 == 0");
    const uintptr_t wa = reinterpret_cast<uintptr_t>(w);
    if (((uintptr_t)x & 3u) || (w_type == HQ_GGML_F32 && (wa & 3u)) || (w_type != HQ_GGML_Q8_0 && (wa & 1u)))
        return fail(HQ_ERR_MISALIGNED, "x must be 4-byte aligned, W aligned to its element");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    cudaError_t e = launch_output_projection(x, static_cast<const uint8_t*>(w), w_type, logits, embedding_dim,
                                             vocab_size, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "output projection launch");
}

HQ_API hq_status hq_embedding_lookup(const void* table, int w_type, int token_id, float* out, int embedding_dim,
                                     int vocab_size, hq_stream_t stream) {
    if (!table || !out) return fail(HQ_ERR_INVALID_ARG, "null pointer argument");
    if (embedding_dim <= 0 || vocab_size <= 0) return fail(HQ_ERR_INVALID_ARG, "bad size");
    if (token_id < 0 || token_id >= vocab_size)
        return fail(HQ_ERR_INVALID_ARG, "token_id %d outside [0, %d)", token_id, vocab_size);
    const bool tq1 = w_type == HQ_GGML_TQ1_0 || w_type == HQ_GGML_TQ1_0_ALT;
    if (w_type != HQ_GGML_F32 && w_type != HQ_GGML_BF16 && w_type != HQ_GGML_Q8_0 && !tq1)
        return fail(HQ_ERR_INVALID_ARG, "w_type %d is not F32 (0), Q8_0 (8), BF16 (30) or TQ1_0 (34, 143)", w_type);
    if ((w_type == HQ_GGML_Q8_0 && embedding_dim % 32) || (tq1 && embedding_dim % 256))
        return fail(HQ_ERR_UNSUPPORTED_SHAPE, "embedding_dim must hold whole blocks");
    const uintptr_t ta = reinterpret_cast<uintptr_t>(table);
    if ((w_type == HQ_GGML_F32 && (ta & 3u)) || (w_type == HQ_GGML_BF16 && (ta & 1u)))
        return fail(HQ_ERR_MISALIGNED, "table not aligned to its element");
    int dev = 0;
    hq_status st = check_device(&dev);
    if (st != HQ_OK) return st;
    cudaError_t e = launch_embedding_lookup(static_cast<const uint8_t*>(table), tq1 ? HQ_GGML_TQ1_0 : w_type, token_id,
                                            out, embedding_dim, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? HQ_OK : cuda_fail(e, "embedding lookup launch");
}

HQ_API void hq_set_launch_overlap(int enable) { set_decode_launch_overlap(enable != 0); }

HQ_API hq_status hq_check_device_error(void) {
    unsigned code = 0;
    cudaError_t e = read_and_clear_device_error(&code);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
    if (code == kDevTimeout) return fail(HQ_ERR_TIMEOUT, "a kernel gave up waiting on a barrier (device timeout)");
    return HQ_OK;
}

}  // extern "C"
