// hq_allreduce.cu -- in-place sum of a 16-bit vector over the GPUs of one
// node, through peer memory over NVLink (the all-reduce that follows the
// row-parallel O and down GEMMs of a tensor-parallel layer).
//
// The reference has no multi-GPU path; this is the collective of the
// Megatron-style split of the quantized linear stack.  Every rank holds its
// partial result in a buffer that all ranks can address (peer-mapped memory,
// e.g. PyTorch symmetric memory); one kernel per rank:
//   1. barrier: rank r stores `epoch` into slot [0][r] of every rank's flag
//      area (system-scope release) and waits until its own slots [0][*] all
//      reach `epoch` (acquire): every partial is complete;
//   2. reduce-scatter + push: rank r sums slice r of the vector over all ranks'
//      buffers and stores the result into slice r of every rank's buffer.
//      With an NVLink multicast address (NVLS) one multimem.ld_reduce per 16
//      bytes returns the sum over all GPUs (fp32 accumulation in the switch)
//      and one multimem.st writes it to every GPU: each rank moves 2/W of the
//      vector.  Without one, 16-byte peer loads from every rank (two vectors in
//      flight per thread and rank) are summed in fp32 in rank order 0..W-1 and
//      stored to every rank: each rank moves 2 (W-1)/W of the vector.  Either
//      way every rank ends with the same bits;
//   3. barrier on slots [1][*] once all of this rank's CTAs have pushed (a
//      counter in the flag area picks the last CTA): every slice has arrived.
// The epoch of a call is either passed in or, with epoch 0, read from that
// counter (it grows by the CTA count per call), so a call can be captured in a
// CUDA graph and replayed.
// Every wait is bounded (kWaitBudgetNs): on time-out the kernel records
// kDevTimeout in the device error word and returns; the result is then
// undefined but no GPU is left spinning.
#include "hq.h"
#include "hq_common.cuh"
#include "hq_internal.h"

#include <cstdio>
#include <type_traits>

namespace hq {

namespace {

constexpr int kArThreads = 512;
constexpr int kArMaxWorld = 8;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until flags[slot*W + j] >= epoch for every rank j (one thread).
__device__ bool wait_all(const unsigned* flags, int slot, int world, unsigned epoch, unsigned* err) {
    const unsigned long long t0 = globaltimer_ns();
    for (int j = 0; j < world; ++j) {
        while ((int)(ld_acquire_sys(flags + slot * kArMaxWorld + j) - epoch) < 0) {
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                record_error(err, kDevTimeout);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

template <typename T>
__device__ __forceinline__ void add8(float (&acc)[8], uint4 v);

template <>
__device__ __forceinline__ void add8<__nv_bfloat16>(float (&acc)[8], uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[2 * i] += __uint_as_float(w[i] << 16);
        acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

template <>
__device__ __forceinline__ void add8<__half>(float (&acc)[8], uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
    }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&acc)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<T, __half>::value) {
            const __half2 h = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
            const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

struct ArParams {
    void* mc;                      // NVLink multicast address of the buffers, or null
    void* bufs[kArMaxWorld];       // each rank's buffer, as addressable from this GPU
    unsigned* flags[kArMaxWorld];  // each rank's flag area: [2][kArMaxWorld] slots + a CTA counter
    int world, rank;
    size_t vecs;  // 16-byte vectors in the buffer
    unsigned epoch;
    unsigned* err;
};

template <typename T>
__global__ void __launch_bounds__(kArThreads) allreduce_kernel(const __grid_constant__ ArParams p) {
    __shared__ int s_ok;
    __shared__ unsigned s_epoch;
    unsigned* my_flags = p.flags[p.rank];
    unsigned* counter = my_flags + 2 * kArMaxWorld;
    // 0. the epoch: given, or derived from this rank's CTA arrival counter, which
    // every earlier call on these flags (same CTA count) raised by gridDim.x, and
    // which CTAs of this call raise only after step 1 (fewer than gridDim.x of
    // them before any CTA of this call reads it): epoch = counter / CTAs + 1.
    if (threadIdx.x == 0) s_epoch = p.epoch ? p.epoch : atomicAdd(counter, 0u) / gridDim.x + 1u;
    __syncthreads();
    const unsigned epoch = s_epoch;
    // 1. every partial is written (each rank's previous kernels have finished)
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) {
            __threadfence_system();
            for (int j = 0; j < p.world; ++j) st_release_sys(p.flags[j] + 0 * kArMaxWorld + p.rank, epoch);
        }
        s_ok = wait_all(my_flags, 0, p.world, epoch, p.err) ? 1 : 0;
    }
    __syncthreads();

    // 2. this rank's slice: sum over ranks in order, push to every rank.  After a
    // timed-out barrier (error word set) the pushes are skipped, but the CTA still
    // counts itself in step 3, so the arrival counter stays in step with the epoch
    // and the next call on these flags is not wedged.
    if (s_ok) {
    const size_t per = (p.vecs + p.world - 1) / p.world;
    const size_t v0 = (size_t)p.rank * per;
    const size_t v1 = v0 + per < p.vecs ? v0 + per : p.vecs;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    if (p.mc) {
        uint4* mc = reinterpret_cast<uint4*>(p.mc);
        for (size_t v = v0 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < v1; v += stride) {
            uint4 r;
            if constexpr (std::is_same<T, __half>::value)
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                             : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                             : "l"(mc + v)
                             : "memory");
            else
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                             : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                             : "l"(mc + v)
                             : "memory");
            asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + v), "r"(r.x),
                         "r"(r.y), "r"(r.z), "r"(r.w)
                         : "memory");
        }
    } else {
        for (size_t v = v0 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < v1; v += 2 * stride) {
            const bool two = v + stride < v1;
            uint4 in[2][kArMaxWorld];
#pragma unroll
            for (int j = 0; j < kArMaxWorld; ++j) {  // L2-only loads: never a stale L1 line of peer memory
                if (j < p.world) {
                    in[0][j] = __ldcg(reinterpret_cast<const uint4*>(p.bufs[j]) + v);
                    if (two) in[1][j] = __ldcg(reinterpret_cast<const uint4*>(p.bufs[j]) + v + stride);
                }
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (h == 1 && !two) break;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < kArMaxWorld; ++j)
                    if (j < p.world) add8<T>(acc, in[h][j]);
                const uint4 out = pack8<T>(acc);
#pragma unroll
                for (int j = 0; j < kArMaxWorld; ++j)
                    if (j < p.world) reinterpret_cast<uint4*>(p.bufs[j])[v + h * stride] = out;
            }
        }
    }

    }

    // 3. the last CTA of this rank to finish its pushes tells every rank; all wait
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned done = atomicAdd(counter, 1u) + 1u;
        if (done == epoch * gridDim.x) {  // every CTA's pushes are ordered before this point
            __threadfence_system();
            for (int j = 0; j < p.world; ++j) st_release_sys(p.flags[j] + 1 * kArMaxWorld + p.rank, epoch);
        }
        if (s_ok) wait_all(my_flags, 1, p.world, epoch, p.err);
    }
}

}  // namespace

}  // namespace hq

extern "C" HQ_API hq_status hq_allreduce_sum(void* const* peer_bufs, unsigned* const* peer_flags, void* multicast,
                                             int world, int rank, hq_dtype dtype, size_t count, unsigned epoch,
                                             int ctas, hq_stream_t stream) {
    using namespace hq;
    if (world < 1 || world > kArMaxWorld || rank < 0 || rank >= world || !peer_bufs || !peer_flags || ctas < 1 ||
        ctas > 1024) {
        set_last_error("hq_allreduce_sum: bad world/rank/pointers/epoch/ctas");
        return HQ_ERR_INVALID_ARG;
    }
    if (dtype != HQ_BF16 && dtype != HQ_F16) {
        set_last_error("hq_allreduce_sum: dtype must be HQ_BF16 or HQ_F16");
        return HQ_ERR_INVALID_ARG;
    }
    if ((count * 2) % 16 != 0) {
        set_last_error("hq_allreduce_sum: count * element size must be a multiple of 16 bytes");
        return HQ_ERR_UNSUPPORTED_SHAPE;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_last_error("hq_allreduce_sum: cudaGetDevice failed");
        return HQ_ERR_CUDA;
    }
    ArParams p{};
    for (int j = 0; j < world; ++j) {
        if (!peer_bufs[j] || !peer_flags[j] || (reinterpret_cast<uintptr_t>(peer_bufs[j]) & 15u)) {
            set_last_error("hq_allreduce_sum: null or misaligned peer pointer");
            return HQ_ERR_MISALIGNED;
        }
        p.bufs[j] = peer_bufs[j];
        p.flags[j] = peer_flags[j];
    }
    if (multicast && (reinterpret_cast<uintptr_t>(multicast) & 15u)) {
        set_last_error("hq_allreduce_sum: misaligned multicast address");
        return HQ_ERR_MISALIGNED;
    }
    p.mc = multicast;
    p.world = world;
    p.rank = rank;
    p.vecs = count * 2 / 16;
    p.epoch = epoch;
    p.err = device_error_word(dev);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == HQ_BF16)
        allreduce_kernel<__nv_bfloat16><<<ctas, kArThreads, 0, s>>>(p);
    else
        allreduce_kernel<__half><<<ctas, kArThreads, 0, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        char buf[128];
        snprintf(buf, sizeof buf, "hq_allreduce_sum launch: %s", cudaGetErrorString(e));
        set_last_error(buf);
        return HQ_ERR_CUDA;
    }
    return HQ_OK;
}
