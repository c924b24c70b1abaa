// ecu_pipe.cuh -- mbarrier + bulk-copy primitives (sm_90+/sm_100a PTX) and
// bounded waits.  Every wait gives up after wait_limit_ns() of wall time, sets
// ECU_STATUS_TIMEOUT in the context's status word and lets the kernel run to
// its end, so that a logic error can never leave a GPU spinning.
#pragma once
#include "ecu_common.cuh"

#ifndef ECU_WAIT_NS
#define ECU_WAIT_NS 2000000000ull   // 2 s: the default limit
#endif

// The wall-time limit of every bounded wait in this translation unit's
// kernels, per device; ecu_set_wait_ns changes it between launches (tests of
// the give-up path shorten it).  Read through the read-only path: it only
// changes while no kernel runs.
static __device__ unsigned long long g_wait_ns = ECU_WAIT_NS;

__device__ __forceinline__ unsigned long long wait_limit_ns() { return __ldg(&g_wait_ns); }

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_init_fence()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe: has phase `parity` of `bar` completed?
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, at most wait_limit_ns().
// Returns false (and flags *status) on timeout.  With FAIL_FAST, a wait that
// finds the step already flagged (by any wait) gives up at once: a kernel
// with thousands of waits then ends after one timeout, not one per wait.
template <bool FAIL_FAST = false>
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *status)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        const uint64_t dt = globaltimer_ns() - t0;
        // the status word is global memory: look at it only once a wait has
        // lasted long enough to suggest trouble, not on every pass
        if (FAIL_FAST && status && dt > 20000 && *reinterpret_cast<volatile int *>(status) != 0) return false;
        if (dt > wait_limit_ns()) {
            if (status) atomicOr(status, ECU_STATUS_TIMEOUT);
            return false;
        }
    }
}

// Wait for a CTA's own bulk copies before it exits, whatever the status word
// says; gives up after limit_ns.
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity, uint64_t limit_ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// One bulk (non-tensor, non-multicast) copy global -> this CTA's shared
// memory, completing `bytes` of transaction count on `bar`.  Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Named barrier among the first `nthreads` threads (multiple of 32).
__device__ __forceinline__ void named_bar(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
