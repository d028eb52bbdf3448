// device_common.cuh — sm_100a device helpers shared by the KV kernels:
// shared-memory mbarriers, 1-D bulk async copies (cp.async.bulk, no
// multicast), an L2 evict-first policy for streamed KV, bounded waits that
// report through a device error flag instead of hanging, and small bit
// helpers.  Hand-written inline PTX; no library code.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace tqkv {

// Device-wide failure flag (first nonzero code wins).  Written by a kernel
// whose bounded wait ran out; read and cleared by tqkv_read_device_error().
// The library keeps all device code in one translation unit, which owns it.
static __device__ unsigned int g_device_error = 0;

enum DeviceErrorCode : unsigned int {
    kErrNone = 0,
    kErrFullWaitTimeout = 1,     // consumer waited too long for a tile
    kErrEmptyWaitTimeout = 2,    // producer waited too long for a free stage
    kErrDrainTimeout = 3,        // producer's copies never completed
    kErrPeerWaitTimeout = 4,     // a peer GPU's exchange entries never arrived
    kErrPieceWaitTimeout = 5,    // a piece of a head split across CTAs never arrived
};

__device__ __forceinline__ void record_device_error(unsigned int code) {
    atomicCAS(&g_device_error, 0u, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Programmatic dependent launch.  launch_dependents lets the next launch in
// the stream (if it was launched as a programmatic dependent) be dispatched
// before this grid completes; wait blocks the calling thread until the grids
// this one depends on have completed and their memory is visible.  Both do
// nothing for a launch without that relation.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Spin on an mbarrier phase with a hard bound.  Returns false (and the caller
// must record an error and leave) when ~2^31 SM cycles (about a second) pass
// without the phase completing.  Normal waits finish in microseconds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
#pragma unroll 1
    for (uint32_t it = 0; it < (1u << 30); ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - start > (1ll << 31)) break;
    }
    return false;
}

// Relaxed 64-bit global accesses at GPU scope (one CTA's stores, another
// CTA's loads; every value carries its own presence tag, so no fences).
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_relaxed_u64x2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];"
                 : "=l"(v.x), "=l"(v.y)
                 : "l"(p)
                 : "memory");
    return v;
}

// L2 policy for data that is read exactly once per step (the KV stream).
__device__ __forceinline__ uint64_t make_evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// 1-D bulk async copy global -> this CTA's shared memory, completing `bytes`
// of transaction count on `bar`.  dst, src and bytes must be multiples of 16.
// No multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Hint: bring [src, src + bytes) into L2 (src and bytes multiples of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrive at a named barrier without waiting for it.
__device__ __forceinline__ void named_barrier_arrive(int id, int nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 2^x, hardware approximation (MUFU.EX2), flush-to-zero; ex2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Integer dot product of four signed bytes of `a` with four signed bytes of
// `b`, plus c.
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Four unsigned bytes of `a` times four signed bytes of `b`, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t float_to_half_bits_rn(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

}  // namespace tqkv
