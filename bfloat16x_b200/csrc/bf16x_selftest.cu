// bf16x_selftest.cu -- runs the library's bounded waits against a barrier or
// flag that nothing completes, so a test can check, without faulting or
// hanging the GPU, that a wait which runs out returns, records the timeout in
// the device status word and leaves the context usable.
#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_status.cuh"
#include "bf16x_wait.cuh"

namespace bf16x {

// which: 0 = mbar_wait (the GEMV's ring slots), 1 = role_wait (the tcgen05
// GEMMs' warp roles), 2 = counter_wait (the slab GEMM's cross-CTA counters),
// 3 = ll_wait (the collective GEMV epilogue's exchange words).  The mbarrier
// is fresh, so its phase 0 never completes; 2 waits for the u32 `*flag` to
// reach 1, 3 for the 64-bit word at `flag` to carry epoch 1 in its high half.
// result[0] = 1 if the wait gave up, result[1] = the abort flag afterwards,
// result[2] = microseconds spent waiting.
__global__ void selftest_wait_kernel(int which, uint64_t limit_ns, const uint32_t *flag, int32_t *result) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
    }
    fence_mbar_init();
    __syncthreads();
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    if (which == 0) ok = mbar_wait(&bar, 0u, &g_status, limit_ns);
    else if (which == 1) ok = role_wait(&bar, 0u, &abort_flag, limit_ns);
    else if (which == 2) ok = counter_wait(flag, 1u, &abort_flag, limit_ns);
    else {
        uint32_t data = 0;
        ok = ll_wait(reinterpret_cast<const uint64_t *>(flag), 1u, data, limit_ns);
    }
    result[0] = ok ? 0 : 1;
    result[1] = abort_flag;
    result[2] = (int32_t)((globaltimer_ns() - t0) / 1000u);
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_selftest_wait(int which, int64_t limit_ns, const uint32_t *flag, int32_t *result, void *stream) {
    if (which < 0 || which > 3) return set_error(BF16X_ERR_INVALID, "bf16x_selftest_wait: which must be 0..3");
    if (limit_ns < 1000 || limit_ns > 100000000)
        return set_error(BF16X_ERR_INVALID, "bf16x_selftest_wait: limit must be 1 us .. 100 ms");
    if (!result || (which >= 2 && !flag)) return set_error(BF16X_ERR_INVALID, "bf16x_selftest_wait: null pointer");
    selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(which, (uint64_t)limit_ns, flag, result);
    return check_launch("selftest_wait_kernel");
}
