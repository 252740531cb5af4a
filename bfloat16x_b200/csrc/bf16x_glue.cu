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

// One CTA per row: h = x (+ delta), y = h * rsqrt(mean(h^2) + eps) * w.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const uint16_t *__restrict__ x,
                                                          const uint16_t *__restrict__ delta,
                                                          const uint16_t *__restrict__ w, float eps, int64_t n,
                                                          uint16_t *__restrict__ h_out, uint16_t *__restrict__ y) {
    const int64_t r = blockIdx.x;
    const uint16_t *xr = x + r * n;
    const uint16_t *dr = delta ? delta + r * n : nullptr;
    __shared__ float red[32];
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        float v = bf(xr[i]);
        if (dr) {
            const uint16_t hb = tobf(v + bf(dr[i]));       // the residual sum is a bf16 tensor
            v = bf(hb);
            h_out[r * n + i] = hb;
        }
        ss += v * v;
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
    const uint16_t *hr = dr ? h_out + r * n : xr;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) y[r * n + i] = tobf(bf(hr[i]) * inv * bf(w[i]));
}

// One CTA per token (b, t): rotate the token's q heads and k heads (pairs
// (2i, 2i+1) of each head by the angle of position pos0 + t) and write q to
// q_out [tokens][H][D], k and v to the cache at [b][pos0 + t].
__global__ void __launch_bounds__(128) rope_qkv_kernel(const uint16_t *__restrict__ qkv, int T, int H, int KV, int D,
                                                       const int64_t *__restrict__ pos0, const float *__restrict__ cos_t,
                                                       const float *__restrict__ sin_t, uint16_t *__restrict__ q_out,
                                                       uint16_t *__restrict__ cache_k, uint16_t *__restrict__ cache_v,
                                                       int64_t cache_ld_b, int64_t max_pos) {
    const int64_t tok = blockIdx.x;
    const int b = (int)(tok / T), t = (int)(tok % T);
    const int64_t pos = *pos0 + t;
    if (pos < 0 || pos >= max_pos) {                      // positions come from device memory: checked here
        if (threadIdx.x == 0) atomicOr(&g_status, kErrBadIndex);
        return;
    }
    const int half = D / 2;
    const uint16_t *src = qkv + tok * (int64_t)(H + 2 * KV) * D;
    uint16_t *kc = cache_k + b * cache_ld_b + pos * (int64_t)KV * D;
    uint16_t *vc = cache_v + b * cache_ld_b + pos * (int64_t)KV * D;
    const int pairs = (H + KV) * half;
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
        const int head = p / half, i = p % half;
        const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
        const float x1 = bf(src[head * D + 2 * i]), x2 = bf(src[head * D + 2 * i + 1]);
        const uint16_t a = tobf(x1 * c - x2 * s), bb = tobf(x1 * s + x2 * c);
        if (head < H) {
            q_out[(tok * H + head) * D + 2 * i] = a;
            q_out[(tok * H + head) * D + 2 * i + 1] = bb;
        } else {
            kc[(head - H) * D + 2 * i] = a;
            kc[(head - H) * D + 2 * i + 1] = bb;
        }
    }
    for (int e = threadIdx.x; e < KV * D; e += blockDim.x) vc[e] = src[(H + KV) * D + e];
}

// out[r][i] = bf16(bf16(silu(gate)) * up) with gate = gu[r][i], up = gu[r][F + i].
__global__ void silu_mul_kernel(const uint16_t *__restrict__ gu, int64_t rows, int64_t F, uint16_t *__restrict__ out) {
    const int64_t n = rows * F;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / F, i = e - r * F;
        const float g = bf(gu[r * 2 * F + i]);
        const float sg = bf(tobf(g / (1.f + expf(-g))));
        out[e] = tobf(sg * bf(gu[r * 2 * F + F + i]));
    }
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_add_rmsnorm(const uint16_t *x, const uint16_t *delta, const uint16_t *w, float eps, int64_t rows,
                                 int64_t n, uint16_t *h_out, uint16_t *y, void *stream) {
    if (rows < 0 || n <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_add_rmsnorm: bad shape");
    if (rows == 0) return BF16X_OK;
    if (!x || !w || !y || (delta && !h_out)) return set_error(BF16X_ERR_INVALID, "bf16x_add_rmsnorm: null pointer");
    if (rows > 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_add_rmsnorm: too many rows");
    add_rmsnorm_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(x, delta, w, eps, n, h_out, y);
    return check_launch("add_rmsnorm_kernel");
}

extern "C" int bf16x_rope_qkv(const uint16_t *qkv, int64_t tokens, int T, int H, int KV, int D, const int64_t *pos0,
                              const float *cos_t, const float *sin_t, uint16_t *q_out, uint16_t *cache_k,
                              uint16_t *cache_v, int64_t cache_ld_b, int64_t max_pos, void *stream) {
    if (tokens < 0 || T <= 0 || H <= 0 || KV <= 0 || D <= 0 || (D & 1) || tokens % T)
        return set_error(BF16X_ERR_INVALID, "bf16x_rope_qkv: bad shape");
    if (tokens == 0) return BF16X_OK;
    if (!qkv || !pos0 || !cos_t || !sin_t || !q_out || !cache_k || !cache_v)
        return set_error(BF16X_ERR_INVALID, "bf16x_rope_qkv: null pointer");
    rope_qkv_kernel<<<(unsigned)tokens, 128, 0, (cudaStream_t)stream>>>(qkv, T, H, KV, D, pos0, cos_t, sin_t, q_out,
                                                                       cache_k, cache_v, cache_ld_b, max_pos);
    return check_launch("rope_qkv_kernel");
}

extern "C" int bf16x_silu_mul(const uint16_t *gu, int64_t rows, int64_t F, uint16_t *out, void *stream) {
    if (rows < 0 || F <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_silu_mul: bad shape");
    if (rows == 0) return BF16X_OK;
    if (!gu || !out) return set_error(BF16X_ERR_INVALID, "bf16x_silu_mul: null pointer");
    const int64_t n = rows * F;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
    silu_mul_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(gu, rows, F, out);
    return check_launch("silu_mul_kernel");
}
