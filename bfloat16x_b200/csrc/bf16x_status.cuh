// bf16x_status.cuh -- per-translation-unit device status word and the host
// helpers every C-ABI entry point uses to report errors.
//
// Each .cu file that includes this header owns one `g_status` word in device
// memory; its kernels OR error bits into it (never trap).  A static
// registration hooks the word into bf16x_device_status(), which reads and
// clears all of them.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <cuda_runtime.h>

#include "../../include/bf16x_b200.h"

namespace bf16x {

static __device__ uint32_t g_status;

// Host side (defined in bf16x_capi.cu).
int set_error(int code, const char *fmt, ...);
void register_status_reader(int (*reader)(uint32_t *));

inline int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return BF16X_OK;
}

namespace {
int read_and_clear_status(uint32_t *flags) {
    uint32_t v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    if (v) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "status clear: %s", cudaGetErrorString(e));
    }
    *flags |= v;
    return BF16X_OK;
}
struct StatusRegistrar {
    StatusRegistrar() { register_status_reader(&read_and_clear_status); }
};
static StatusRegistrar g_status_registrar;
}  // namespace

}  // namespace bf16x
