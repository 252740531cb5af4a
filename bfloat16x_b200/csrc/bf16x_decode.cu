// bf16x_decode.cu -- flat-stream decode with the overflow fix fused in.
//
// Replaces the reference's two-kernel decode (_bf16x_decode_kernel +
// _bf16x_fix_ovf_kernel, bf16x_triton_test.py:11-108) and its host-side
// filter/.item() sync with one pass:
//   * a CTA owns a tile of 8192 consecutive flat elements, one 32-element
//     group per thread: 1 sign word, 7 mantissa words, 3 delta words and two
//     emax bytes, all whole words because the group is 32-aligned;
//   * two warps locate the tile's slice of the sorted overflow table with a
//     32-ary search while the others decode;
//   * the tile is assembled in shared memory, the slice is applied there
//     (only at positions whose stream delta is the saturated 7, which is the
//     reference decode's rule, opqk_linear.py:367-372), and the tile leaves
//     with coalesced 16-byte stores.
#include "bf16x_common.cuh"
#include "bf16x_flat.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

constexpr int kDecThreads = 256;
constexpr int kDecTile = kDecThreads * 32;   // elements per CTA

__global__ void __launch_bounds__(kDecThreads)
flat_decode_kernel(FlatStreams f, uint16_t *__restrict__ out) {
    __shared__ __align__(16) uint32_t tile[kDecTile / 2];    // bf16 pairs
    __shared__ int64_t slice[2];

    const int tid = threadIdx.x;
    const int64_t t0 = (int64_t)blockIdx.x * kDecTile;
    const int64_t t1 = min(t0 + (int64_t)kDecTile, f.n);
    const int warp = tid >> 5;

    if (warp < 2 && f.n_ovf > 0) {
        const int64_t r = warp_lower_bound(f.ovf_idx, f.n_ovf, warp == 0 ? t0 : t1);
        if ((tid & 31) == 0) slice[warp] = r;
    }

    // ---- base decode of this thread's 32-element group
    const int64_t g = (int64_t)blockIdx.x * kDecThreads + tid;   // global group index
    const int64_t e0 = g * 32;
    if (e0 < f.n) {
        uint32_t sw, mw[8], dw[4];
        uint32_t eb0, eb1;
        const bool full = (g + 1) * 7 <= f.n_mant && (g + 1) * 3 <= f.n_delta &&
                          g < f.n_sign && 2 * g + 1 < f.n_emax;
        if (full) {
            sw = __ldg(f.sign + g);
#pragma unroll
            for (int i = 0; i < 7; ++i) mw[i] = __ldg(f.mant + 7 * g + i);
#pragma unroll
            for (int i = 0; i < 3; ++i) dw[i] = __ldg(f.delta + 3 * g + i);
            eb0 = __ldg(f.emax + 2 * g);
            eb1 = __ldg(f.emax + 2 * g + 1);
        } else {
            sw = ld_word(f.sign, f.n_sign, g);
#pragma unroll
            for (int i = 0; i < 7; ++i) mw[i] = ld_word(f.mant, f.n_mant, 7 * g + i);
#pragma unroll
            for (int i = 0; i < 3; ++i) dw[i] = ld_word(f.delta, f.n_delta, 3 * g + i);
            eb0 = 2 * g < f.n_emax ? __ldg(f.emax + 2 * g) : 0u;
            eb1 = 2 * g + 1 < f.n_emax ? __ldg(f.emax + 2 * g + 1) : 0u;
        }
        mw[7] = 0u;
        dw[3] = 0u;
        uint32_t pairs[16];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t s = (sw >> i) & 1u;
            const uint32_t mb = 7 * i, db = 3 * i;
            const uint32_t m = funnel_r(mw[mb >> 5], mw[(mb >> 5) + 1], mb & 31) & 0x7Fu;
            const uint32_t d = funnel_r(dw[db >> 5], dw[(db >> 5) + 1], db & 31) & 0x7u;
            const uint32_t e = i < 16 ? eb0 : eb1;
            const uint32_t b = (s << 15) | (((e - d) & 0xFFu) << 7) | m;
            if (i & 1) pairs[i >> 1] |= b << 16; else pairs[i >> 1] = b;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(tile + tid * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pairs[4 * i], pairs[4 * i + 1], pairs[4 * i + 2], pairs[4 * i + 3]);
    }
    __syncthreads();

    // ---- overflow fix inside shared memory
    if (f.n_ovf > 0) {
        const int64_t lo = slice[0], hi = slice[1];
        uint16_t *t16 = reinterpret_cast<uint16_t *>(tile);
        for (int64_t j = lo + tid; j < hi; j += kDecThreads) {
            const int64_t pos = __ldg(f.ovf_idx + j);
            if (j > 0 && (int64_t)__ldg(f.ovf_idx + j - 1) >= pos) atomicOr(&g_status, kErrOvfUnsorted);
            if (pos < t0 || pos >= t1) { atomicOr(&g_status, kErrOvfRange); continue; }
            const uint32_t val = __ldg(f.ovf_val + j);
            const int64_t ei = pos / 16;
            const uint32_t e = ei < f.n_emax ? __ldg(f.emax + ei) : 0u;
            const uint32_t cur = t16[pos - t0];
            // the reference substitutes the table delta only where the stream says 7
            if (((cur >> 7) & 0xFFu) == ((e - 7u) & 0xFFu))
                t16[pos - t0] = (uint16_t)((cur & 0x807Fu) | (((e - val) & 0xFFu) << 7));
        }
        // entries outside every tile (index >= N) are found by the last CTA
        if (blockIdx.x == gridDim.x - 1 && tid == 0 && hi < f.n_ovf) atomicOr(&g_status, kErrOvfRange);
        if (blockIdx.x == 0 && tid == 0 && f.n_ovf > 0 && __ldg(f.ovf_idx) < 0) atomicOr(&g_status, kErrOvfRange);
        __syncthreads();
    }

    // ---- coalesced store
    const int64_t cnt = t1 - t0;
    if (cnt == kDecTile) {
        const uint4 *src = reinterpret_cast<const uint4 *>(tile);
        uint4 *dst = reinterpret_cast<uint4 *>(out + t0);
        for (int i = tid; i < kDecTile / 8; i += kDecThreads) dst[i] = src[i];
    } else {
        const uint16_t *src = reinterpret_cast<const uint16_t *>(tile);
        for (int64_t i = tid; i < cnt; i += kDecThreads) out[t0 + i] = src[i];
    }
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_decode(const uint32_t *sign, int64_t n_sign_words,
                            const uint32_t *mant, int64_t n_mant_words,
                            const uint32_t *delta, int64_t n_delta_words,
                            const uint8_t *emax, int64_t n_emax,
                            const int32_t *ovf_idx, const uint8_t *ovf_val, int64_t n_ovf,
                            int64_t out_f, int64_t in_f, int sub,
                            uint16_t *out, void *stream) {
    if (out_f < 0 || in_f < 0) return set_error(BF16X_ERR_INVALID, "bf16x_decode: negative shape");
    if (sub != 16) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_decode: only sub=16 is supported");
    const int64_t n = out_f * in_f;
    if (n == 0) return BF16X_OK;
    if (!sign || !mant || !delta || !emax || !out)
        return set_error(BF16X_ERR_INVALID, "bf16x_decode: null stream pointer");
    if (n_ovf < 0 || (n_ovf > 0 && (!ovf_idx || !ovf_val)))
        return set_error(BF16X_ERR_INVALID, "bf16x_decode: bad overflow table");
    if (n_sign_words < (n + 31) / 32 || n_mant_words < (7 * n + 31) / 32 ||
        n_delta_words < (3 * n + 31) / 32 || n_emax < (n + 15) / 16)
        return set_error(BF16X_ERR_INVALID, "bf16x_decode: stream shorter than out_f*in_f elements need");
    if (reinterpret_cast<uintptr_t>(out) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_decode: out must be 16-byte aligned");
    FlatStreams f{sign, n_sign_words, mant, n_mant_words, delta, n_delta_words,
                  emax, n_emax, ovf_idx, ovf_val, n_ovf, n};
    const int64_t grid = (n + kDecTile - 1) / kDecTile;
    if (grid > 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_decode: tensor too large");
    flat_decode_kernel<<<(unsigned)grid, kDecThreads, 0, (cudaStream_t)stream>>>(f, out);
    return check_launch("bf16x_decode");
}
