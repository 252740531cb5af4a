// bf16x_glue.cu -- the element-wise glue between the projections of the
// end-to-end Llama-style decoder used to measure the hot path in a model
// (bfloat16x_b200/llama_e2e.py): residual add + RMSNorm, rotary embedding of
// q and k together with the write of k and v into the static KV cache, and
// SiLU(gate) * up.  The reference has no decoder of its own; these replace a
// few dozen tiny framework kernels per layer (each a launch of a couple of
// microseconds at batch 1) by three, so the decode step's time goes to the
// weight-streaming GEMVs.  All arithmetic is fp32 with bf16 rounding at the
// points where the framework version rounds.
#include <algorithm>

#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t tobf(float f) { return f32_to_bf16_bits_rn(f); }

// The glue kernels sit between the decoder's GEMVs.  Each lets the next
// kernel of the stream launch as soon as it starts (so a GEMV requests its
// weights while the glue runs) and, launched itself as a dependent, waits for
// the previous kernel only before reading its inputs.

constexpr int kNormThreads = 512;
constexpr int kNormVec = 8;                    // bf16 per 16-byte access

// One CTA per row: h = x (+ delta), y = h * rsqrt(mean(h^2) + eps) * w.  Rows
// of up to kNormThreads * kNormVec elements (8192) stay in registers between
// the two passes; longer rows are read twice.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const uint16_t *__restrict__ x,
                                                                  const uint16_t *__restrict__ delta,
                                                                  const uint16_t *__restrict__ w, float eps, int64_t n,
                                                                  uint16_t *__restrict__ h_out,
                                                                  uint16_t *__restrict__ y) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t r = blockIdx.x;
    const uint16_t *xr = x + r * n;
    const uint16_t *dr = delta ? delta + r * n : nullptr;
    __shared__ float red[kNormThreads / 32];
    const bool vec = (n % kNormVec) == 0 && n <= (int64_t)kNormThreads * kNormVec &&
                     ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(dr) |
                       reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y + r * n) |
                       reinterpret_cast<uintptr_t>(h_out ? h_out + r * n : nullptr)) & 15u) == 0;
    float v[kNormVec];
    float ss = 0.f;
    const int64_t i0 = (int64_t)threadIdx.x * kNormVec;
    if (vec) {
        if (i0 < n) {
            const uint4 a = *reinterpret_cast<const uint4 *>(xr + i0);
            const uint16_t *ah = reinterpret_cast<const uint16_t *>(&a);
            uint4 hv;
            uint16_t *hh = reinterpret_cast<uint16_t *>(&hv);
            if (dr) {
                const uint4 dd = *reinterpret_cast<const uint4 *>(dr + i0);
                const uint16_t *dh = reinterpret_cast<const uint16_t *>(&dd);
#pragma unroll
                for (int k = 0; k < kNormVec; ++k) {
                    hh[k] = tobf(bf(ah[k]) + bf(dh[k]));    // the residual sum is a bf16 tensor
                    v[k] = bf(hh[k]);
                }
                *reinterpret_cast<uint4 *>(h_out + r * n + i0) = hv;
            } else {
#pragma unroll
                for (int k = 0; k < kNormVec; ++k) v[k] = bf(ah[k]);
            }
#pragma unroll
            for (int k = 0; k < kNormVec; ++k) ss += v[k] * v[k];
        }
    } else {
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
            float t = bf(xr[i]);
            if (dr) {
                const uint16_t hb = tobf(t + bf(dr[i]));
                t = bf(hb);
                h_out[r * n + i] = hb;
            }
            ss += t * t;
        }
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)n + eps);
    if (vec) {
        if (i0 < n) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(w + i0);
            const uint16_t *wh = reinterpret_cast<const uint16_t *>(&wv);
            uint4 o;
            uint16_t *oh = reinterpret_cast<uint16_t *>(&o);
#pragma unroll
            for (int k = 0; k < kNormVec; ++k) oh[k] = tobf(v[k] * inv * bf(wh[k]));
            *reinterpret_cast<uint4 *>(y + r * n + i0) = o;
        }
    } else {
        const uint16_t *hr = dr ? h_out + r * n : xr;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) y[r * n + i] = tobf(bf(hr[i]) * inv * bf(w[i]));
    }
}

// One CTA per (token, head) of q and k, plus one per token for v: rotate the
// head's pairs (2i, 2i+1) by the angle of position pos0 + t; q to q_out
// [tokens][H][D], k and v to the cache at [b][pos0 + t].
__global__ void __launch_bounds__(64) rope_qkv_kernel(const uint16_t *__restrict__ qkv, int T, int H, int KV, int D,
                                                      const int64_t *__restrict__ pos0, const float *__restrict__ cos_t,
                                                      const float *__restrict__ sin_t, uint16_t *__restrict__ q_out,
                                                      uint16_t *__restrict__ cache_k, uint16_t *__restrict__ cache_v,
                                                      int64_t cache_ld_b, int64_t max_pos) {
    griddep_launch_dependents();
    griddep_wait();
    const int per_tok = H + KV + 1;
    const int64_t tok = blockIdx.x / per_tok;
    const int head = blockIdx.x % per_tok;
    const int b = (int)(tok / T), t = (int)(tok % T);
    const int64_t pos = *pos0 + t;
    if (pos < 0 || pos >= max_pos) {                      // positions come from device memory: checked here
        if (threadIdx.x == 0) atomicOr(&g_status, kErrBadIndex);
        return;
    }
    const int half = D / 2;
    const uint16_t *src = qkv + tok * (int64_t)(H + 2 * KV) * D;
    if (head == H + KV) {                                 // v: copied into the cache
        uint16_t *vc = cache_v + b * cache_ld_b + pos * (int64_t)KV * D;
        for (int e = threadIdx.x; e < KV * D; e += blockDim.x) vc[e] = src[(H + KV) * D + e];
        return;
    }
    uint16_t *dst = head < H ? q_out + (tok * H + head) * D
                             : cache_k + b * cache_ld_b + pos * (int64_t)KV * D + (head - H) * D;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
        const uint32_t pr = *reinterpret_cast<const uint32_t *>(src + head * D + 2 * i);
        const float x1 = bf((uint16_t)(pr & 0xFFFFu)), x2 = bf((uint16_t)(pr >> 16));
        const uint32_t o = (uint32_t)tobf(x1 * c - x2 * s) | ((uint32_t)tobf(x1 * s + x2 * c) << 16);
        *reinterpret_cast<uint32_t *>(dst + 2 * i) = o;
    }
}

// out[r][i] = bf16(bf16(silu(gate)) * up) with gate = gu[r][i], up = gu[r][F + i].
__global__ void silu_mul_kernel(const uint16_t *__restrict__ gu, int64_t rows, int64_t F, uint16_t *__restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t n = rows * F;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / F, i = e - r * F;
        const float g = bf(gu[r * 2 * F + i]);
        const float sg = bf(tobf(g / (1.f + expf(-g))));
        out[e] = tobf(sg * bf(gu[r * 2 * F + F + i]));
    }
}

// Launch as a programmatic dependent of the previous kernel of the stream.
template <typename... KArgs, typename... Args>
static int launch_dependent(void (*kern)(KArgs...), unsigned grid, unsigned block, cudaStream_t st, const char *what,
                            Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "%s: launch: %s", what, cudaGetErrorString(e));
    return check_launch(what);
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_add_rmsnorm(const uint16_t *x, const uint16_t *delta, const uint16_t *w, float eps, int64_t rows,
                                 int64_t n, uint16_t *h_out, uint16_t *y, void *stream) {
    if (rows < 0 || n <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_add_rmsnorm: bad shape");
    if (rows == 0) return BF16X_OK;
    if (!x || !w || !y || (delta && !h_out)) return set_error(BF16X_ERR_INVALID, "bf16x_add_rmsnorm: null pointer");
    if (rows > 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_add_rmsnorm: too many rows");
    return launch_dependent(add_rmsnorm_kernel, (unsigned)rows, kNormThreads, (cudaStream_t)stream, "add_rmsnorm_kernel",
                            x, delta, w, eps, n, h_out, y);
}

extern "C" int bf16x_rope_qkv(const uint16_t *qkv, int64_t tokens, int T, int H, int KV, int D, const int64_t *pos0,
                              const float *cos_t, const float *sin_t, uint16_t *q_out, uint16_t *cache_k,
                              uint16_t *cache_v, int64_t cache_ld_b, int64_t max_pos, void *stream) {
    if (tokens < 0 || T <= 0 || H <= 0 || KV <= 0 || D <= 0 || (D & 1) || tokens % T)
        return set_error(BF16X_ERR_INVALID, "bf16x_rope_qkv: bad shape");
    if (tokens == 0) return BF16X_OK;
    if (!qkv || !pos0 || !cos_t || !sin_t || !q_out || !cache_k || !cache_v)
        return set_error(BF16X_ERR_INVALID, "bf16x_rope_qkv: null pointer");
    if (tokens * (H + KV + 1) > 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_rope_qkv: too many tokens");
    return launch_dependent(rope_qkv_kernel, (unsigned)(tokens * (H + KV + 1)), 64, (cudaStream_t)stream,
                            "rope_qkv_kernel", qkv, T, H, KV, D, pos0, cos_t, sin_t, q_out, cache_k, cache_v,
                            cache_ld_b, max_pos);
}

extern "C" int bf16x_silu_mul(const uint16_t *gu, int64_t rows, int64_t F, uint16_t *out, void *stream) {
    if (rows < 0 || F <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_silu_mul: bad shape");
    if (rows == 0) return BF16X_OK;
    if (!gu || !out) return set_error(BF16X_ERR_INVALID, "bf16x_silu_mul: null pointer");
    const int64_t n = rows * F;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
    return launch_dependent(silu_mul_kernel, (unsigned)grid, 256, (cudaStream_t)stream, "silu_mul_kernel", gu, rows, F,
                            out);
}
