// hq_common.cuh -- shared device helpers for the sm_100a quantized-linear kernels:
// mbarrier / bulk-copy / tcgen05 / mma.sync wrappers (inline PTX), the fused
// int4 and ternary register dequantisers, bounded waits and the device error word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hq {

// ------------------------------------------------------------------ errors
// Kernels never spin forever: a wait that exceeds kWaitBudgetNs records a code
// in the device error word (a __device__ variable of hq_api.cu whose address
// every launch passes in) and the kernel winds down.  Read and cleared by
// hq_check_device_error().
enum DevError : unsigned { kDevOk = 0, kDevTimeout = 1 };

constexpr unsigned long long kWaitBudgetNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(unsigned* err, unsigned code) {
    if (err) atomicExch(err, code);
}

// ----------------------------------------------------------------- address
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// try_wait: the hardware parks a waiting thread for a short, system-defined
// time and wakes it when the phase completes.  No suspend-time hint: a long
// hint measurably delays the wake-up after the phase completes on B200
// (~1-2 us per stage in a streaming ring), which a producer / consumer
// pipeline pays on every stage.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: true on success, false (and the device error word set) on timeout.
// try_wait parks the thread in hardware until the phase completes (or a short
// system-defined limit passes), so polling it costs almost no issue slots and
// wakes the warp as soon as the data lands.  A software sleep between polls
// (__nanosleep) would add its wake-up granularity to every stage a consumer
// reaches before its data -- in a streaming kernel, nearly every stage.  The
// clock is read once per 64 polls to enforce kWaitBudgetNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
            record_error(err, kDevTimeout);
            return false;
        }
    }
}

// --------------------------------------------------------------- bulk copy
// 1-D bulk copy global -> shared (TMA engine), completion via mbarrier tx bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 cache policy (createpolicy) for the source lines.
__device__ __forceinline__ void bulk_g2s_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 16-byte asynchronous copy global -> shared through the load/store path
// (L2 only).  Small operands go this way rather than through the TMA engine,
// which charges a fixed cost per bulk operation.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the arrival is counted in the barrier's expected count: no increment).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 2-D tiled TMA load of box {x, y} (x innermost, in elements) from a tensor map
// held in kernel parameter space; completion via mbarrier tx bytes.  x times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---------------------------------------------------- clusters and PDL
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of all CTAs of the cluster; release/acquire orders shared-memory
// writes before the barrier with distributed-shared-memory reads after it.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Programmatic dependent launch: let the next kernel on the stream start its
// prologue now / wait until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ loads
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Read-only 16-byte load through L1 (activations: small, reused by every warp).
__device__ __forceinline__ uint4 ldg128_nc(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// ---------------------------------------------------------------- lop3/prmt
template <uint32_t LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return d;
}
// (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    return lop3<(0xF0 & 0xCC) | 0xAA>(a, b, c);
}

// ---------------------------------------------------------------- types
template <typename T>
struct TypeTraits;
template <>
struct TypeTraits<__half> {
    static constexpr bool is_bf16 = false;
};
template <>
struct TypeTraits<__nv_bfloat16> {
    static constexpr bool is_bf16 = true;
};

__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

// --------------------------------------------------------------- dequant
// Code fields are placed so that codes of k and k+1 sit 16 bits apart (see the
// tile layout in hq_layout.h).  OR-ing a field into the mantissa of a
// floating-point constant M yields the exact value M + code ("raw" values).
// The exact dequantisers subtract M + offset with one packed op; the raw ones
// skip it: the decode kernel feeds raw values straight into the MMA and
// removes M + offset through a per-block activation row sum (an MMA with a
// constant A operand that starts the accumulator).
//
// int4 word: pairs (e0,e1) (e2,e3) live in the low nibble of each byte
// (nibbles 0/4 and 2/6), (e4,e5) (e6,e7) in the high nibble (1/5 and 3/7).
// Outputs are in k order: o[0]=(e0,e1) o[1]=(e2,e3) o[2]=(e4,e5) o[3]=(e6,e7).

// fp16, raw.  o[0], o[1] = 1024 + u; o[2], o[3] = 1024 + 16 u (high-nibble
// class, masked in place: the 1/16 goes onto the activation operand instead).
__device__ __forceinline__ void raw_u4_f16(uint32_t w, uint32_t (&o)[4]) {
    const uint32_t kMagic = 0x64006400u;  // 1024.0 in both halves
    const uint32_t w8 = w >> 8;
    o[0] = and_or(w, 0x000F000Fu, kMagic);
    o[1] = and_or(w8, 0x000F000Fu, kMagic);
    o[2] = and_or(w, 0x00F000F0u, kMagic);
    o[3] = and_or(w8, 0x00F000F0u, kMagic);
}

// bf16, raw: 128 + u for all four pairs (bf16 has no room for the 16u form).
__device__ __forceinline__ void raw_u4_bf16(uint32_t w, uint32_t (&o)[4]) {
    const uint32_t kMagic = 0x43004300u;  // 128.0
    o[0] = and_or(w, 0x000F000Fu, kMagic);
    o[1] = and_or(w >> 8, 0x000F000Fu, kMagic);
    o[2] = and_or(w >> 4, 0x000F000Fu, kMagic);
    o[3] = and_or(w >> 12, 0x000F000Fu, kMagic);
}

// fp16, exact: q = u - 8 (or the code u itself when kUnsigned).
template <bool kUnsigned = false>
__device__ __forceinline__ void dequant_u4_f16(uint32_t w, uint32_t (&o)[4]) {
    const uint32_t kSubLo = kUnsigned ? 0x64006400u : 0x64086408u;  // 1024 (+8)
    const uint32_t kMulHi = 0x2C002C00u;                             // 1/16
    const uint32_t kAddHi = kUnsigned ? 0xD400D400u : 0xD480D480u;  // -64 (-72)
    uint32_t r[4];
    raw_u4_f16(w, r);
    asm("sub.f16x2 %0, %1, %2;" : "=r"(o[0]) : "r"(r[0]), "r"(kSubLo));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(o[1]) : "r"(r[1]), "r"(kSubLo));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[2]) : "r"(r[2]), "r"(kMulHi), "r"(kAddHi));
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(o[3]) : "r"(r[3]), "r"(kMulHi), "r"(kAddHi));
}

// bf16, exact.
template <bool kUnsigned = false>
__device__ __forceinline__ void dequant_u4_bf16(uint32_t w, uint32_t (&o)[4]) {
    const uint32_t kSub = kUnsigned ? 0x43004300u : 0x43084308u;  // 128 (+8)
    uint32_t r[4];
    raw_u4_bf16(w, r);
#pragma unroll
    for (int i = 0; i < 4; ++i) asm("sub.bf16x2 %0, %1, %2;" : "=r"(o[i]) : "r"(r[i]), "r"(kSub));
}

// ternary: pair p (codes of k=2p, 2p+1) sits at bits (2p, 16+2p); raw = M + c.
template <bool kBF16>
__device__ __forceinline__ uint32_t raw_t2_pair(uint32_t w, int p) {
    return and_or(w >> (2 * p), 0x00030003u, kBF16 ? 0x43004300u : 0x64006400u);
}

// ternary, exact: t = c - 1.
template <bool kBF16>
__device__ __forceinline__ uint32_t dequant_t2_pair(uint32_t w, int p) {
    const uint32_t kSub = kBF16 ? 0x43014301u : 0x64016401u;  // constant + 1
    uint32_t a = raw_t2_pair<kBF16>(w, p);
    uint32_t o;
    if (kBF16)
        asm("sub.bf16x2 %0, %1, %2;" : "=r"(o) : "r"(a), "r"(kSub));
    else
        asm("sub.f16x2 %0, %1, %2;" : "=r"(o) : "r"(a), "r"(kSub));
    return o;
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// ----------------------------------------------- column gather (tile order)
// The codes of one output column c = g + 8 hh of a 64-k chunk (tile order, see
// hq_layout.h) live in the fragments of lanes 4g .. 4g+3, 16 k each.  A thread
// that owns column c (tensor-memory operand layout: one column per lane) reads
// the four fragments starting at a rotated lane, `rot`, chosen so that the 16
// threads of a half-warp (int4, 8-byte loads) or the 32 threads of a warp
// (ternary, 4-byte loads) touch distinct banks; the rotation is then undone in
// registers.  Output: the column's words in k order, w[i] = k 8i .. 8i+7 (int4)
// or k 16i .. 16i+15 (ternary).
template <typename T>
__device__ __forceinline__ void unrotate4(T (&v)[4], int rot) {
    // v[j] holds fragment (j + rot) & 3; afterwards v[t] holds fragment t.
    if (rot & 1) {
        const T a = v[3];
        v[3] = v[2];
        v[2] = v[1];
        v[1] = v[0];
        v[0] = a;
    }
    if (rot & 2) {
        T a = v[0];
        v[0] = v[2];
        v[2] = a;
        a = v[1];
        v[1] = v[3];
        v[3] = a;
    }
}

// int4: rot = g >> 1 (lane = 16 s' + 8 hh + g within the warp).
__device__ __forceinline__ void gather_column_u4(const uint8_t* chunk, int g, int hh, int rot, bool valid,
                                                 uint32_t (&w)[8]) {
    uint2 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        v[j] = valid ? *reinterpret_cast<const uint2*>(chunk + (4 * g + ((j + rot) & 3)) * 16 + 8 * hh)
                     : make_uint2(0u, 0u);
    unrotate4(v, rot);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        w[2 * t] = v[t].x;
        w[2 * t + 1] = v[t].y;
    }
}

// ternary: rot = (g >> 2) + 2 s' (lane = 16 s' + 8 hh + g within the warp).
__device__ __forceinline__ void gather_column_t2(const uint8_t* chunk, int g, int hh, int rot, bool valid,
                                                 uint32_t (&w)[4]) {
    uint32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        v[j] = valid ? *reinterpret_cast<const uint32_t*>(chunk + (4 * g + ((j + rot) & 3)) * 8 + 4 * hh) : 0u;
    unrotate4(v, rot);
#pragma unroll
    for (int t = 0; t < 4; ++t) w[t] = v[t];
}

// ------------------------------------------------------------- tcgen05
// Tensor-memory allocation (one warp, .sync.aligned), MMA issue (one thread),
// completion commits to mbarriers, and TMEM -> register loads.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle (8-row x 128 B
// atoms stacked every 1024 B), tile base 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
    uint64_t d = (uint64_t)((smem_addr & 0x3FFFFu) >> 4);  // start address
    d |= (uint64_t)1 << 16;                                // leading byte offset (16 B units; unused for K-major SW128)
    d |= (uint64_t)(1024 >> 4) << 32;                      // stride byte offset: 8-row atom pitch
    d |= (uint64_t)1 << 46;                                // descriptor version (sm100)
    d |= (uint64_t)2 << 61;                                // layout: SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A/B K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(bool bf16, int M, int N) {
    return (1u << 4)                        // D format: f32
           | ((bf16 ? 1u : 0u) << 7)        // A format
           | ((bf16 ? 1u : 0u) << 10)       // B format
           | ((uint32_t)(N >> 3) << 17)     // N / 8
           | ((uint32_t)(M >> 4) << 24);    // M / 16
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 8 registers -> 32 lanes x 8 consecutive 32-bit columns (thread i = lane i of
// the warp's quadrant).  The address is warp-uniform: every thread passes the
// same lane/column base.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (tensor memory) [+]= A (tensor memory: row m in lane m, k-pairs in
// consecutive 32-bit columns) x B (shared-memory descriptor).  One thread issues.
// ---------------------------------------------- CTA pairs (cta_group::2)
// Two CTAs of a cluster (ranks 0 and 1) run one MMA of M = 256: each holds
// 128 rows of A and of the accumulator in its own tensor memory and N/2 rows
// of B in its own shared memory; rank 0 issues it.  No multicast loads.
// Arrive on the barrier at the same offset in CTA `rank` (default semantics; a
// tcgen05.fence::before_thread_sync before it orders this thread's tensor-memory
// stores ahead of the consumer's tcgen05 work).  A release at cluster scope
// here costs a memory barrier per arrive: measured as the kernel's top stall.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, %1;\n\t"
        "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
        "r"(rank)
        : "memory");
}
// 2-D TMA load into this CTA's shared memory whose completion (bytes) is
// counted on a barrier of either CTA of the pair (shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[256 x N] (+)= A[256 x 16] (tensor memory of both CTAs) x B[16 x N] (N/2 rows
// from each CTA's shared memory at the descriptor's address).
__device__ __forceinline__ void umma_ts_f16_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
            d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}
// Arrive on the barrier at this offset in every CTA of `cta_mask` when the
// pair's MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(smem_u32(bar)), "h"(cta_mask) : "memory");
}

__device__ __forceinline__ void umma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// ------------------------------------------------------------- mma.sync
// D = A * B + C with separate C and D registers (no copy of a shared seed).
template <bool kBF16>
__device__ __forceinline__ void mma_16816_c(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                            const float (&c)[4]) {
    if (kBF16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
              "f"(c[3]));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%10,%11,%12,%13};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
              "f"(c[3]));
    }
}

// D(16x8,f32) += A(16x16) * B(16x8), fp16 or bf16 inputs.
template <bool kBF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    // Plain (non-volatile) asm: a pure register operation the compiler may
    // schedule freely, so independent MMA chains interleave.
    if (kBF16) {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

}  // namespace hq
