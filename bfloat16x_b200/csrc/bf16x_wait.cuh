// bf16x_wait.cuh -- the bounded waits of the kernels whose warps or CTAs wait
// on one another (the tcgen05 GEMMs' warp roles, the slab GEMM's cross-CTA
// counters, the GEMV's collective epilogue).
//
// Every wait gives up after `limit_ns` of %globaltimer (kWaitLimitNs, 2 s, in
// the kernels), sets kErrWaitTimeout in this translation unit's status word
// and raises the caller's abort flag, so a broken pipeline or a peer that
// never arrives ends the kernel with an error the host reads back
// (bf16x_device_status) instead of hanging the GPU.  The limit is a
// parameter so the self-test entry point (bf16x_selftest_wait) can run these
// very functions against a barrier or flag nobody completes with a short one.
#pragma once

#include "bf16x_common.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

// Bounded mbarrier wait used by every GEMM role; on timeout the abort flag is
// raised and false is returned, and a role that finds the flag raised while
// waiting gives up too.
// The fast path (phase already complete) reads nothing else: the abort flag
// is a shared-memory load, and on the MMA issuer's path one such load per
// wait measurably slows the issue of the k-blocks.  It is checked while
// waiting instead.
__device__ __forceinline__ bool role_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (*abort_flag) return false;
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 7u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            atomicOr(&g_status, kErrWaitTimeout);
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Wait until *ctr >= target (another CTA's progress); bounded like role_wait.
__device__ __forceinline__ bool counter_wait(const uint32_t *ctr, uint32_t target, volatile int *abort_flag,
                                             uint64_t limit_ns = kWaitLimitNs) {
    if (ld_acquire_gpu(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (*abort_flag) return false;
        __nanosleep(64);
        if (ld_acquire_gpu(ctr) >= target) return true;
        if ((i & 15u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            atomicOr(&g_status, kErrWaitTimeout);
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Wait until the 64-bit exchange word *w (written by this or another GPU in
// one single-copy-atomic store: data in the low half, launch epoch in the
// high half) carries `epoch`; *data gets its low half.  Bounded like the others.
__device__ __forceinline__ bool ll_wait(const uint64_t *w, uint32_t epoch, uint32_t &data,
                                        uint64_t limit_ns = kWaitLimitNs) {
    uint64_t v = ld_relaxed_sys_u64(w);
    if ((uint32_t)(v >> 32) == epoch) { data = (uint32_t)v; return true; }
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(32);
        v = ld_relaxed_sys_u64(w);
        if ((uint32_t)(v >> 32) == epoch) { data = (uint32_t)v; return true; }
        if ((i & 15u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            atomicOr(&g_status, kErrWaitTimeout);
            data = 0u;
            return false;
        }
    }
}

}  // namespace bf16x
