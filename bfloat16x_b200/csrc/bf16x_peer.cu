// bf16x_peer.cu -- device memory shared with the other GPUs of one node over
// NVLink (CUDA IPC), for the collective epilogue of bf16x_gemv_peers.
//
// Every rank exports a buffer of its own (an allocation made by its host
// framework); the handles travel between processes over the host side of
// the process group; every rank maps its peers' buffers into its address
// space, so a kernel can store straight into another GPU's memory.
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

static MemGetAddressRangeFn address_range_fn() {
    static MemGetAddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<MemGetAddressRangeFn>(p);
    });
    return fn;
}

// Opened peer allocations, by handle bytes: the mapping and how many imports
// share it (a handle can be mapped once per process).
struct Opened {
    void *base;
    int refs;
};
static std::map<std::string, Opened> &opened() {
    static std::map<std::string, Opened> m;
    return m;
}
static std::mutex &opened_mu() {
    static std::mutex mu;
    return mu;
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int64_t bf16x_peer_handle_bytes(void) { return (int64_t)sizeof(cudaIpcMemHandle_t); }

extern "C" int bf16x_peer_export(const void *ptr, void *handle, int64_t *offset) {
    if (!ptr || !handle || !offset) return set_error(BF16X_ERR_INVALID, "bf16x_peer_export: null pointer");
    MemGetAddressRangeFn fn = address_range_fn();
    if (!fn) return set_error(BF16X_ERR_CUDA, "bf16x_peer_export: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return set_error(BF16X_ERR_INVALID, "bf16x_peer_export: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_peer_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    std::memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return BF16X_OK;
}

extern "C" int bf16x_peer_import(const void *handle, void **base) {
    if (!handle || !base) return set_error(BF16X_ERR_INVALID, "bf16x_peer_import: null pointer");
    const std::string key(static_cast<const char *>(handle), sizeof(cudaIpcMemHandle_t));
    std::lock_guard<std::mutex> lk(opened_mu());
    auto it = opened().find(key);
    if (it != opened().end()) {
        ++it->second.refs;
        *base = it->second.base;
        return BF16X_OK;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_peer_import: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    opened()[key] = Opened{p, 1};
    *base = p;
    return BF16X_OK;
}

extern "C" int bf16x_peer_close(void *base) {
    std::lock_guard<std::mutex> lk(opened_mu());
    for (auto it = opened().begin(); it != opened().end(); ++it) {
        if (it->second.base != base) continue;
        if (--it->second.refs == 0) {
            cudaError_t e = cudaIpcCloseMemHandle(base);
            opened().erase(it);
            if (e != cudaSuccess)
                return set_error(BF16X_ERR_CUDA, "bf16x_peer_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
        }
        return BF16X_OK;
    }
    return set_error(BF16X_ERR_INVALID, "bf16x_peer_close: not an imported peer buffer");
}
