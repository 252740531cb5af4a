// bf16x_capi.cu -- library-level entry points: version, error strings and the
// device status registry.
#include <mutex>
#include <string>
#include <vector>

#include "bf16x_common.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

static thread_local std::string t_last_error;

int set_error(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

static std::vector<int (*)(uint32_t *)> &readers() {
    static std::vector<int (*)(uint32_t *)> r;
    return r;
}
static std::mutex &readers_mu() {
    static std::mutex m;
    return m;
}

void register_status_reader(int (*reader)(uint32_t *)) {
    std::lock_guard<std::mutex> lk(readers_mu());
    readers().push_back(reader);
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_version(void) { return 1; }

extern "C" const char *bf16x_last_error(void) { return t_last_error.c_str(); }

extern "C" int bf16x_device_status(int device, uint32_t *flags) {
    if (!flags) return set_error(BF16X_ERR_INVALID, "bf16x_device_status: null flags");
    *flags = 0;
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if ((e = cudaSetDevice(device)) != cudaSuccess)
        return set_error(BF16X_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    int rc = BF16X_OK;
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) {
        rc = set_error(BF16X_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
    } else {
        std::lock_guard<std::mutex> lk(readers_mu());
        for (auto fn : readers()) {
            rc = fn(flags);
            if (rc != BF16X_OK) break;
        }
    }
    cudaSetDevice(prev);
    return rc;
}
