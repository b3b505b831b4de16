// sa_ptx.cuh -- thin inline-PTX wrappers for the sm_100a features the kernels
// use: mbarriers, bulk (TMA) copies, tensor-map copies, exp2, and a bounded
// wait that reports a timeout instead of spinning forever.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace sa {

// Device-side waits give up after this many nanoseconds of %globaltimer and
// record SA_STATUS_TIMEOUT in the context's status word.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

enum : int { SA_STATUS_OK = 0, SA_STATUS_TIMEOUT = 1, SA_STATUS_BAD_INDEX = 2 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for the phase with `parity` to complete.  Returns false (and records a
// timeout in *status when non-null) if it has not completed within the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) {
            if (status) atomicExch(status, SA_STATUS_TIMEOUT);
            return false;
        }
    }
    return true;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Same with an L2 eviction-priority hint (policy from createpolicy).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// launch now, and (in a kernel launched with programmatic serialization) wait
// until the previous kernel has completed and its writes are visible.  Both
// are no-ops for kernels launched the ordinary way.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Self-validating exchange words between GPUs: (epoch << 32) | 32 value bits,
// written with one 8-byte store, so a reader that sees the epoch also sees
// the value (aligned 8-byte accesses are single-copy atomic).  System scope:
// the writer may be another GPU storing over NVLink.
__device__ __forceinline__ void st_u64_relaxed_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_u64_relaxed_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long epoch_word(unsigned epoch, float x) {
    return ((unsigned long long)epoch << 32) | __float_as_uint(x);
}
// Wait (bounded, as mbar_wait) until the word at p carries `epoch`; return
// its value.  After an earlier expired wait (*status set) it does not wait
// again, so one missing peer costs one limit, not one per word.
__device__ __forceinline__ float wait_epoch_word(const unsigned long long* p, unsigned epoch, int* status) {
    unsigned long long w = ld_u64_relaxed_sys(p);
    if ((unsigned)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
    if (*reinterpret_cast<volatile int*>(status) != 0) return __uint_as_float((uint32_t)w);
    const unsigned long long t0 = globaltimer();
    while ((unsigned)((w = ld_u64_relaxed_sys(p)) >> 32) != epoch) {
        if (globaltimer() - t0 > kWaitLimitNs) {
            atomicExch(status, SA_STATUS_TIMEOUT);
            break;
        }
    }
    return __uint_as_float((uint32_t)w);
}

// 2^x on the SFU (MUFU.EX2), flush-to-zero; 2^-inf = 0.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace sa
