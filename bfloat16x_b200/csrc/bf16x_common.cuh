// bf16x_common.cuh -- shared device helpers for the BF16X sm_100a kernels.
//
// Everything here is hand-written PTX / CUDA for Blackwell (sm_100a):
// mbarrier-based pipelines fed by the bulk-copy (TMA) engine, bounded waits
// that report a timeout instead of hanging, and the bit tricks shared by the
// decoders.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "../../include/bf16x_b200.h"

namespace bf16x {

// Device-side status bits (OR-ed into a per-translation-unit status word and
// read back by bf16x_device_status()).
enum : uint32_t {
    kErrWaitTimeout   = 1u << 0,   // an mbarrier wait gave up
    kErrOvfUnsorted   = 1u << 1,   // overflow index not strictly ascending
    kErrOvfRange      = 1u << 2,   // overflow index outside [0, N)
    kErrBadLayout     = 1u << 3,   // resident layout inconsistent with its arguments
    kErrBadIndex      = 1u << 4,   // a device-side index (a decoder position) out of range
};

// Upper bound for one mbarrier wait, in nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Raise the barrier's expected transaction bytes without arriving (the
// arrival comes later, with the rest of the phase's copies).
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Programmatic dependent launch.  launch_dependents lets the next kernel of
// the stream (launched with programmatic stream serialization) be scheduled
// as this grid's CTAs retire; wait blocks until the previous kernel of the
// stream has completed and its writes are visible.  Without a dependent
// launch both are no-ops.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// try_wait with a suspend-time hint: a waiting warp sleeps (up to the hint)
// instead of spinning, so it does not take issue slots from working warps.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// limit_ns (kWaitLimitNs in the kernels), sets kErrWaitTimeout in *status and
// returns false, so a broken pipeline ends the kernel with an error instead of
// hanging the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *status,
                                          uint64_t limit_ns = kWaitLimitNs) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(a, parity)) return true;
        if ((i & 7u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            atomicOr(status, kErrWaitTimeout);
            return false;
        }
    }
}

// ------------------------------------------------------------- bulk copies
// 1-D bulk copy global -> shared (TMA engine), completion counted in bytes on
// an mbarrier.  src and dst must be 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst_smem)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// ------------------------------------------------------------ small helpers
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t funnel_r(uint32_t lo, uint32_t hi, uint32_t sh) {
    return __funnelshift_r(lo, hi, sh);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) {
    return __uint_as_float(b16 << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits_rn(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

template <int SH>
__device__ __forceinline__ uint32_t shl_signed(uint32_t v) {
    if constexpr (SH >= 0) return v << SH; else return v >> (-SH);
}

}  // namespace bf16x

// ------------------------------------------------------- tensor-map copies
namespace bf16x {

// Tiled TMA loads into this CTA's shared memory, completion counted on an
// mbarrier.  `map` is the address of a __grid_constant__ kernel parameter.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const void *map, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const void *map, int c0, int c1, int c2, int c3,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
        :: "r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)) : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses with later
// async-proxy ones (TMA writes, tensor-core reads) of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const void *map) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(map) : "memory");
}

}  // namespace bf16x
