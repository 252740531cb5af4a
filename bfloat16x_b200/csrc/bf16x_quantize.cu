// bf16x_quantize.cu -- GPU packer producing the bf16x_quantize dict.
//
// Device counterpart of bf16x_quantize (opqk_linear.py:291-324), bit for bit:
//   emax[j]   = max exponent of flat elements [16j, 16j+16) (zero padded),
//   delta     = emax - exponent; entries with delta >= 7 go to the overflow
//               table (ascending flat index, true delta) and the stream holds 7,
//   streams   = LSB-first int32 words with the reference's lengths
//               (pack_bits_stream pads the value list, opqk_linear.py:53-64).
// A thread packs one 32-element group: 1 sign word, 7 mantissa words and 3
// delta words, all whole words.  Two passes: count (per-CTA totals into the
// scratch, then an exclusive scan) and encode (ordered table writes).
#include "bf16x_common.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

constexpr int kQThreads = 256;
constexpr int kQTile = kQThreads * 32;

struct Group32 {
    uint32_t sw, mw[7], dw[3];
    uint32_t e0, e1;
    uint32_t ovf_mask;    // bit i: element i has delta >= 7
    uint32_t dval[32];    // true deltas (only read where ovf_mask is set)
};

__device__ __forceinline__ void pack_group(const uint16_t *w, int64_t n, int64_t g, Group32 &G) {
    const int64_t e0 = g * 32;
    const int cnt = (int)(n - e0 < 32 ? n - e0 : 32);
    uint32_t bits[32];
    if (cnt == 32 && ((reinterpret_cast<uintptr_t>(w + e0) & 15u) == 0)) {
        const uint4 *src = reinterpret_cast<const uint4 *>(w + e0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldg(src + i);
            bits[8 * i + 0] = v.x & 0xFFFFu; bits[8 * i + 1] = v.x >> 16;
            bits[8 * i + 2] = v.y & 0xFFFFu; bits[8 * i + 3] = v.y >> 16;
            bits[8 * i + 4] = v.z & 0xFFFFu; bits[8 * i + 5] = v.z >> 16;
            bits[8 * i + 6] = v.w & 0xFFFFu; bits[8 * i + 7] = v.w >> 16;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) bits[i] = i < cnt ? (uint32_t)__ldg(w + e0 + i) : 0u;
    }
    uint32_t em0 = 0, em1 = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const uint32_t ex = (bits[i] >> 7) & 0xFFu;   // padding elements have exponent 0
        if (i < 16) em0 = max(em0, ex); else em1 = max(em1, ex);
    }
    G.e0 = em0;
    G.e1 = em1;
    G.sw = 0;
    G.ovf_mask = 0;
#pragma unroll
    for (int i = 0; i < 7; ++i) G.mw[i] = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) G.dw[i] = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (i >= cnt) break;
        const uint32_t b = bits[i];
        const uint32_t d = (i < 16 ? em0 : em1) - ((b >> 7) & 0xFFu);
        G.dval[i] = d;
        const uint32_t d3 = d >= 7u ? 7u : d;
        if (d >= 7u) G.ovf_mask |= 1u << i;
        G.sw |= ((b >> 15) & 1u) << i;
        const int mb = 7 * i, db = 3 * i;
        G.mw[mb >> 5] |= (b & 0x7Fu) << (mb & 31);
        if ((mb & 31) + 7 > 32) G.mw[(mb >> 5) + 1] |= (b & 0x7Fu) >> (32 - (mb & 31));
        G.dw[db >> 5] |= d3 << (db & 31);
        if ((db & 31) + 3 > 32) G.dw[(db >> 5) + 1] |= d3 >> (32 - (db & 31));
    }
}

__device__ __forceinline__ int block_exclusive_scan(int v, int &total) {
    __shared__ int ws[kQThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) ws[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < kQThreads / 32 ? ws[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < kQThreads / 32) ws[lane] = w;
    }
    __syncthreads();
    total = ws[kQThreads / 32 - 1];
    const int excl = (warp ? ws[warp - 1] : 0) + x - v;
    __syncthreads();
    return excl;
}

__global__ void __launch_bounds__(kQThreads) quantize_count_kernel(const uint16_t *w, int64_t n, int64_t *cta_counts) {
    const int64_t g = (int64_t)blockIdx.x * kQThreads + threadIdx.x;
    int c = 0;
    if (g * 32 < n) {
        Group32 G;
        pack_group(w, n, g, G);
        c = __popc(G.ovf_mask);
    }
    int total = 0;
    block_exclusive_scan(c, total);
    if (threadIdx.x == 0) cta_counts[blockIdx.x] = total;
}

// Exclusive scan of int64 counts in place; a[n] = total, also copied to *out_total.
__global__ void __launch_bounds__(1024) scan64_kernel(int64_t *a, int64_t n, int64_t *out_total) {
    __shared__ int64_t ws[32];
    __shared__ int64_t carry_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += 1024) {
        const int64_t i = base + tid;
        const int64_t v = i < n ? a[i] : 0;
        int64_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) ws[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int64_t s = ws[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            ws[lane] = s;
        }
        __syncthreads();
        const int64_t excl = carry_s + (warp ? ws[warp - 1] : 0) + x - v;
        if (i < n) a[i] = excl;
        __syncthreads();
        if (tid == 1023) carry_s = excl + v;
        __syncthreads();
    }
    if (tid == 0) {
        a[n] = carry_s;
        *out_total = carry_s;
    }
}

__global__ void __launch_bounds__(kQThreads)
quantize_encode_kernel(const uint16_t *w, int64_t n, const int64_t *cta_off, uint8_t *emax, uint32_t *sign,
                       int64_t nw_sign, uint32_t *mant, int64_t nw_mant, uint32_t *delta, int64_t nw_delta,
                       int64_t n_emax, int32_t *ovf_idx, uint8_t *ovf_val, int64_t capacity) {
    const int64_t g = (int64_t)blockIdx.x * kQThreads + threadIdx.x;
    Group32 G;
    int c = 0;
    const bool active = g * 32 < n;
    if (active) {
        pack_group(w, n, g, G);
        c = __popc(G.ovf_mask);
    }
    int total = 0;
    const int excl = block_exclusive_scan(c, total);
    if (!active) return;
    if (g < nw_sign) sign[g] = G.sw;
#pragma unroll
    for (int i = 0; i < 7; ++i)
        if (7 * g + i < nw_mant) mant[7 * g + i] = G.mw[i];
#pragma unroll
    for (int i = 0; i < 3; ++i)
        if (3 * g + i < nw_delta) delta[3 * g + i] = G.dw[i];
    if (2 * g < n_emax) emax[2 * g] = (uint8_t)G.e0;
    if (2 * g + 1 < n_emax) emax[2 * g + 1] = (uint8_t)G.e1;
    int64_t pos = cta_off[blockIdx.x] + excl;
    uint32_t m = G.ovf_mask;
    while (m) {
        const int i = __ffs(m) - 1;
        m &= m - 1;
        if (pos < capacity) {
            ovf_idx[pos] = (int32_t)(g * 32 + i);
            ovf_val[pos] = (uint8_t)G.dval[i];
        }
        ++pos;
    }
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int64_t bf16x_stream_words(int64_t n, int bits) {
    if (n <= 0 || bits <= 0) return 0;
    const int64_t nbits = n * bits;
    const int64_t pad = ((-nbits) % 32 + 32) % 32;   // value padding, opqk_linear.py:55-58
    return ((n + pad) * bits + 31) / 32;
}

extern "C" int64_t bf16x_quantize_scratch_bytes(int64_t n) {
    const int64_t ctas = (n + kQTile - 1) / kQTile;
    return (ctas + 1) * (int64_t)sizeof(int64_t);
}

extern "C" int bf16x_quantize_count(const uint16_t *w, int64_t n, int sub, void *scratch, int64_t *n_ovf_dev,
                                    void *stream) {
    if (sub != 16) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_quantize: only sub=16 is supported");
    if (n < 0) return set_error(BF16X_ERR_INVALID, "bf16x_quantize_count: negative size");
    if (!scratch || !n_ovf_dev) return set_error(BF16X_ERR_INVALID, "bf16x_quantize_count: null scratch/output");
    if (n > 0 && !w) return set_error(BF16X_ERR_INVALID, "bf16x_quantize_count: null input");
    if (n / 32 > 0x7fffffffLL * kQThreads) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_quantize: too large");
    if (n >= 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_quantize: int32 overflow index limits N < 2^31");
    cudaStream_t st = (cudaStream_t)stream;
    int64_t *counts = static_cast<int64_t *>(scratch);
    const int64_t ctas = (n + kQTile - 1) / kQTile;
    if (ctas > 0) {
        quantize_count_kernel<<<(unsigned)ctas, kQThreads, 0, st>>>(w, n, counts);
        int rc = check_launch("quantize_count_kernel");
        if (rc) return rc;
    }
    scan64_kernel<<<1, 1024, 0, st>>>(counts, ctas, n_ovf_dev);
    return check_launch("scan64_kernel");
}

extern "C" int bf16x_quantize(const uint16_t *w, int64_t n, int sub, const void *scratch, uint8_t *emax,
                              uint32_t *sign, uint32_t *mant, uint32_t *delta, int32_t *ovf_idx, uint8_t *ovf_val,
                              int64_t capacity, void *stream) {
    if (sub != 16) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_quantize: only sub=16 is supported");
    if (n < 0 || capacity < 0) return set_error(BF16X_ERR_INVALID, "bf16x_quantize: negative size");
    if (n == 0) return BF16X_OK;
    if (!w || !scratch || !emax || !sign || !mant || !delta)
        return set_error(BF16X_ERR_INVALID, "bf16x_quantize: null pointer");
    if (capacity > 0 && (!ovf_idx || !ovf_val)) return set_error(BF16X_ERR_INVALID, "bf16x_quantize: null table");
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t nw_sign = bf16x_stream_words(n, 1), nw_mant = bf16x_stream_words(n, 7);
    const int64_t nw_delta = bf16x_stream_words(n, 3), n_emax = (n + 15) / 16;
    const int64_t G = (n + 31) / 32;
    // words past the last group exist when the reference's value padding is long
    if (nw_mant > 7 * G) cudaMemsetAsync(mant + 7 * G, 0, (nw_mant - 7 * G) * 4, st);
    if (nw_delta > 3 * G) cudaMemsetAsync(delta + 3 * G, 0, (nw_delta - 3 * G) * 4, st);
    const int64_t ctas = (n + kQTile - 1) / kQTile;
    quantize_encode_kernel<<<(unsigned)ctas, kQThreads, 0, st>>>(
        w, n, static_cast<const int64_t *>(scratch), emax, sign, nw_sign, mant, nw_mant, delta, nw_delta, n_emax,
        ovf_idx, ovf_val, capacity);
    return check_launch("quantize_encode_kernel");
}
