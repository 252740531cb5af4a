// bf16x_gguf.cu -- the GGUF BF16X block format (llama.cpp GGML_TYPE_BF16X)
// and its lossless side table, on the GPU.
//
// Device counterparts of the numpy reference bf16x_gguf_block.py:
//   quantize_blocks   (:64-81)   bf16 -> 46-byte blocks of 32 weights
//   dequantize_blocks (:84-95)   blocks -> bf16 (delta 7 = zero marker)
//   pack_ovf          (:143-161) exact bits of the clamped weights, by row
//   apply_ovf         (:174-181) write them back over a dequantized tensor
//
// Block layout (46 bytes): emax[2] (per 16-weight half, floored at 7),
// sign[4] (1 bit per weight), mant[28] (7 bits), delta[12] (3 bits), every
// bit field LSB-first.  One thread owns one block; the blocks of a CTA and
// their values are staged in shared memory so that global memory is read and
// written with coalesced 4-byte accesses (a block is 46 bytes, a CTA of 128
// blocks 5,888 bytes, a multiple of 16).
#include <algorithm>

#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_gguf.cuh"
#include "bf16x_resident.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

constexpr int kGBlk = 46;          // bytes per block
constexpr int kGCta = 128;         // blocks (threads) per CTA
constexpr int kGPitch = 33;        // staged values per block (32 + 1: conflict-free rows)

// float32 bits -> bf16 bits with the reference's rounding: quiet NaNs keep
// their high half with bit 6 set, everything else rounds to nearest even
// (bf16_gguf_block.py:45-50).
__device__ __forceinline__ uint32_t gguf_f32_to_bf16(uint32_t n) {
    if ((n & 0x7FFFFFFFu) > 0x7F800000u) n = (n & 0xFFFF0000u) | (64u << 16);
    return (uint32_t)(((uint64_t)n + 0x7FFFu + ((n >> 16) & 1u)) >> 16) & 0xFFFFu;
}

// One input element as bf16 bits.  mode: BF16X_DTYPE_BF16 (bits as given),
// BF16X_DTYPE_F32 (round), BF16X_DTYPE_F32_TRUNC (high half, for float32
// values known to be bf16-exact).
__device__ __forceinline__ uint32_t load_bits(const void *x, int64_t i, int mode) {
    if (mode == BF16X_DTYPE_BF16) return reinterpret_cast<const uint16_t *>(x)[i];
    const uint32_t u = reinterpret_cast<const uint32_t *>(x)[i];
    return mode == BF16X_DTYPE_F32 ? gguf_f32_to_bf16(u) : (u >> 16);
}

// ------------------------------------------------------------------ quantize
__global__ void __launch_bounds__(kGCta) gguf_quantize_kernel(const void *x, int mode, int64_t nblocks,
                                                              uint8_t *blocks) {
    __shared__ uint32_t vals[kGCta * kGPitch];
    __shared__ __align__(16) uint8_t out[kGCta * kGBlk];
    const int64_t b0 = (int64_t)blockIdx.x * kGCta;
    const int nb = (int)std::min<int64_t>(kGCta, nblocks - b0);
    for (int i = threadIdx.x; i < nb * 32; i += kGCta)
        vals[(i >> 5) * kGPitch + (i & 31)] = load_bits(x, b0 * 32 + i, mode);
    __syncthreads();
    if (threadIdx.x < nb) {
        const uint32_t *v = vals + threadIdx.x * kGPitch;
        uint32_t emax[2] = {7u, 7u};
#pragma unroll
        for (int j = 0; j < 32; ++j) emax[j >> 4] = max(emax[j >> 4], (v[j] >> 7) & 0xFFu);
        uint32_t sgn = 0, mw[7] = {0, 0, 0, 0, 0, 0, 0}, dw[3] = {0, 0, 0};
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const uint32_t n = v[j], e = (n >> 7) & 0xFFu;
            sgn |= ((n >> 15) & 1u) << j;
            const uint32_t m = n & 0x7Fu;
            const int mp = 7 * j;
            mw[mp >> 5] |= m << (mp & 31);
            if ((mp & 31) > 25) mw[(mp >> 5) + 1] |= m >> (32 - (mp & 31));
            const uint32_t dl = min(emax[j >> 4] - e, 7u);
            const int dp = 3 * j;
            dw[dp >> 5] |= dl << (dp & 31);
            if ((dp & 31) > 29) dw[(dp >> 5) + 1] |= dl >> (32 - (dp & 31));
        }
        // 46 bytes at a 2-byte aligned offset: 23 halfwords
        uint16_t *o = reinterpret_cast<uint16_t *>(out + threadIdx.x * kGBlk);
        o[0] = (uint16_t)(emax[0] | (emax[1] << 8));
        o[1] = (uint16_t)sgn;
        o[2] = (uint16_t)(sgn >> 16);
#pragma unroll
        for (int w = 0; w < 7; ++w) { o[3 + 2 * w] = (uint16_t)mw[w]; o[4 + 2 * w] = (uint16_t)(mw[w] >> 16); }
#pragma unroll
        for (int w = 0; w < 3; ++w) { o[17 + 2 * w] = (uint16_t)dw[w]; o[18 + 2 * w] = (uint16_t)(dw[w] >> 16); }
    }
    __syncthreads();
    const int bytes = nb * kGBlk;
    uint8_t *dst = blocks + b0 * kGBlk;
    const int words = bytes >> 2;
    for (int i = threadIdx.x; i < words; i += kGCta)
        reinterpret_cast<uint32_t *>(dst)[i] = reinterpret_cast<const uint32_t *>(out)[i];
    for (int i = words * 4 + threadIdx.x; i < bytes; i += kGCta) dst[i] = out[i];
}

// ---------------------------------------------------------------- dequantize
__global__ void __launch_bounds__(kGCta) gguf_dequantize_kernel(const uint8_t *blocks, int64_t nblocks,
                                                                void *y, int y_f32) {
    __shared__ __align__(16) uint8_t in[kGCta * kGBlk];
    __shared__ uint32_t vals[kGCta * kGPitch];
    const int64_t b0 = (int64_t)blockIdx.x * kGCta;
    const int nb = (int)std::min<int64_t>(kGCta, nblocks - b0);
    const int bytes = nb * kGBlk, words = bytes >> 2;
    const uint8_t *src = blocks + b0 * kGBlk;
    for (int i = threadIdx.x; i < words; i += kGCta)
        reinterpret_cast<uint32_t *>(in)[i] = reinterpret_cast<const uint32_t *>(src)[i];
    for (int i = words * 4 + threadIdx.x; i < bytes; i += kGCta) in[i] = src[i];
    __syncthreads();
    if (threadIdx.x < nb) {
        const uint16_t *h = reinterpret_cast<const uint16_t *>(in + threadIdx.x * kGBlk);
        const uint32_t em0 = h[0] & 0xFFu, em1 = h[0] >> 8;
        const uint32_t sgn = h[1] | ((uint32_t)h[2] << 16);
        uint32_t mw[8], dw[4];
#pragma unroll
        for (int w = 0; w < 7; ++w) mw[w] = h[3 + 2 * w] | ((uint32_t)h[4 + 2 * w] << 16);
        mw[7] = 0;
#pragma unroll
        for (int w = 0; w < 3; ++w) dw[w] = h[17 + 2 * w] | ((uint32_t)h[18 + 2 * w] << 16);
        dw[3] = 0;
        uint32_t *v = vals + threadIdx.x * kGPitch;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int mp = 7 * j, dp = 3 * j;
            const uint32_t m = __funnelshift_r(mw[mp >> 5], mw[(mp >> 5) + 1], mp & 31) & 0x7Fu;
            const uint32_t dl = __funnelshift_r(dw[dp >> 5], dw[(dp >> 5) + 1], dp & 31) & 0x7u;
            const uint32_t em = j < 16 ? em0 : em1;
            const uint32_t e = dl == 7u ? 0u : (em > dl ? em - dl : 0u);
            v[j] = (((sgn >> j) & 1u) << 15) | (e << 7) | m;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nb * 32; i += kGCta) {
        const uint32_t b = vals[(i >> 5) * kGPitch + (i & 31)];
        if (y_f32) reinterpret_cast<uint32_t *>(y)[b0 * 32 + i] = b << 16;
        else reinterpret_cast<uint16_t *>(y)[b0 * 32 + i] = (uint16_t)b;
    }
}

// ---------------------------------------------------------- overflow table
// Bit j of the result: element j of the 32-column block at x[i0..i0+31] is
// clamped by quantize (true delta >= 7 against the floored half-block max) and
// is not +-0 (zero decodes exactly through the zero marker) --
// bf16x_gguf_block.py:123-131.
__device__ __forceinline__ uint32_t ovf_mask32(const void *x, int64_t i0, int mode, uint32_t (&bits)[32]) {
    uint32_t emax[2] = {7u, 7u};
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        bits[j] = load_bits(x, i0 + j, mode);
        emax[j >> 4] = max(emax[j >> 4], (bits[j] >> 7) & 0xFFu);
    }
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const uint32_t e = (bits[j] >> 7) & 0xFFu;
        if (emax[j >> 4] - e >= 7u && (bits[j] & 0x7FFFu) != 0u) mask |= 1u << j;
    }
    return mask;
}

// One CTA per row (grid-stride): counts[r] = entries of row r.
__global__ void __launch_bounds__(256) gguf_ovf_count_kernel(const void *x, int mode, int64_t rows, int64_t cols,
                                                             uint32_t *counts) {
    __shared__ uint32_t part[8];
    const int64_t nbr = cols / 32;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        uint32_t c = 0;
        for (int64_t b = threadIdx.x; b < nbr; b += blockDim.x) {
            uint32_t bits[32];
            c += __popc(ovf_mask32(x, r * cols + b * 32, mode, bits));
        }
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t s = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += part[w];
            counts[r] = s;
        }
        __syncthreads();
    }
}

// In-place exclusive scan of n values with one CTA (n <= a few million):
// v[0..n) counts -> v[0..n] offsets, v[n] = total.
__global__ void __launch_bounds__(1024) gguf_scan_kernel(uint32_t *v, int64_t n) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const uint32_t x = i < n ? v[i] : 0u;
        uint32_t s = x;
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += t;
        }
        if (lane == 31) warp_sums[w] = s;
        __syncthreads();
        if (w == 0) {
            uint32_t ws = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0u;
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, ws, o);
                if (lane >= o) ws += t;
            }
            warp_sums[lane] = ws;                      // inclusive over warps
        }
        __syncthreads();
        const uint32_t before = carry + (w ? warp_sums[w - 1] : 0u) + s - x;
        if (i < n) v[i] = before;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = before + x;
        __syncthreads();
    }
    if (threadIdx.x == 0) v[n] = carry;
}

// One CTA per row: entries in column order (blocks are visited in order
// b = k*blockDim + tid, each round scanned across the CTA).
__global__ void __launch_bounds__(256) gguf_ovf_pack_kernel(const void *x, int mode, int64_t rows, int64_t cols,
                                                            const uint32_t *row_off, uint16_t *ecols,
                                                            uint16_t *ebits) {
    __shared__ uint32_t warp_sums[8];
    __shared__ uint32_t round_base;
    const int64_t nbr = cols / 32;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        if (threadIdx.x == 0) round_base = row_off[r];
        __syncthreads();
        for (int64_t k0 = 0; k0 < nbr; k0 += blockDim.x) {
            const int64_t b = k0 + threadIdx.x;
            uint32_t bits[32];
            const uint32_t mask = b < nbr ? ovf_mask32(x, r * cols + b * 32, mode, bits) : 0u;
            const uint32_t c = __popc(mask);
            uint32_t s = c;
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += t;
            }
            if (lane == 31) warp_sums[w] = s;
            __syncthreads();
            uint32_t before = round_base + s - c;
            for (int q = 0; q < w; ++q) before += warp_sums[q];
            uint32_t m = mask;
            while (m) {
                const int j = __ffs(m) - 1;
                m &= m - 1;
                ecols[before] = (uint16_t)(b * 32 + j);
                ebits[before] = (uint16_t)bits[j];
                ++before;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                uint32_t t = 0;
                for (int q = 0; q < nw; ++q) t += warp_sums[q];
                round_base += t;
            }
            __syncthreads();
        }
    }
}

// One thread per entry: the row is found by binary search of row_off.
__global__ void gguf_apply_ovf_kernel(void *y, int y_f32, int64_t rows, int64_t cols, const uint32_t *row_off,
                                      const uint16_t *ecols, const uint16_t *ebits, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = 0, hi = rows;                   // row_off[lo] <= i < row_off[hi]
        while (hi - lo > 1) {
            const int64_t mid = (lo + hi) >> 1;
            if ((int64_t)row_off[mid] <= i) lo = mid; else hi = mid;
        }
        const int64_t c = ecols[i];
        if (c >= cols) { atomicOr(&g_status, kErrOvfRange); continue; }
        const int64_t at = lo * cols + c;
        if (y_f32) reinterpret_cast<uint32_t *>(y)[at] = (uint32_t)ebits[i] << 16;
        else reinterpret_cast<uint16_t *>(y)[at] = ebits[i];
    }
}

// ------------------------------------------ side table -> per-item records
// The records the GGUF-block GEMV stages with each (16-row tile, 256-column
// chunk) item (bf16x_gguf.cuh).  One CTA per tile, threads strided over the
// tile's (row, chunk) pairs: a row's entries are sorted by column, so those
// of one chunk are a contiguous range, found by binary search and counted
// per half (block parity).  WRITE = false stores each item's record size in
// words (scanned into offsets afterwards); WRITE = true fills the records,
// entries of half 0 first, each half by row then column, deterministically.
// Row offsets are clamped to [0, n_entries] and columns at or past in_f
// fall in no chunk, so both kernels see the same (possibly clipped) table
// and the writes stay inside the records the counts sized; the counting
// pass reports any such table through the status word.
__device__ __forceinline__ int64_t col_lower_bound(const uint16_t *cols, int64_t lo, int64_t hi, uint32_t v) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((uint32_t)cols[mid] < v) lo = mid + 1; else hi = mid;
    }
    return lo;
}

template <bool WRITE>
__global__ void __launch_bounds__(256) gguf_side_kernel(const uint32_t *row_off, const uint16_t *cols,
                                                        const uint16_t *bits, int64_t rows, int64_t in_f,
                                                        int64_t n_entries, int nch, int32_t *item_off,
                                                        uint32_t *recs) {
    extern __shared__ int32_t side_sh[];
    int32_t *cnt = side_sh;                 // [(c * 16 + r) * 2 + half]
    int32_t *first = side_sh + nch * 32;    // [c * 16 + r]: the range's first entry
    const int64_t r0 = (int64_t)blockIdx.x * kTileRows;
    const int nr = (int)(rows - r0 < kTileRows ? rows - r0 : kTileRows);
    if constexpr (!WRITE) {
        if (blockIdx.x == 0 && threadIdx.x == 0 && (row_off[0] != 0u || (int64_t)row_off[rows] != n_entries))
            atomicOr(&g_status, kErrOvfRange);
        for (int r = threadIdx.x; r < nr; r += blockDim.x) {
            const int64_t b = row_off[r0 + r], e = row_off[r0 + r + 1];
            if (e < b || e > n_entries) { atomicOr(&g_status, kErrOvfRange); continue; }
            for (int64_t k = b; k < e; ++k) {
                if ((int64_t)cols[k] >= in_f) atomicOr(&g_status, kErrOvfRange);
                if (k > b && cols[k - 1] >= cols[k]) atomicOr(&g_status, kErrOvfUnsorted);
            }
        }
    }
    for (int i = threadIdx.x; i < nch * kTileRows; i += blockDim.x) {
        const int c = i >> 4, r = i & 15;
        int32_t n0 = 0, n1 = 0;
        int64_t a = 0;
        if (r < nr) {
            const int64_t e = ::min((int64_t)row_off[r0 + r + 1], n_entries);
            const int64_t b = ::min((int64_t)row_off[r0 + r], e);
            a = col_lower_bound(cols, b, e, 256u * c);
            const int64_t z = col_lower_bound(cols, a, e, 256u * (c + 1));
            for (int64_t k = a; k < z; ++k) {
                if ((cols[k] >> 5) & 1u) ++n1; else ++n0;
            }
        }
        cnt[2 * i] = n0;
        cnt[2 * i + 1] = n1;
        first[i] = (int32_t)a;
    }
    __syncthreads();
    if constexpr (!WRITE) {
        for (int c = threadIdx.x; c < nch; c += blockDim.x) {
            int32_t n = 0;
            for (int r = 0; r < kTileRows; ++r) n += cnt[2 * (c * 16 + r)] + cnt[2 * (c * 16 + r) + 1];
            item_off[(int64_t)blockIdx.x * nch + c] = (int32_t)gguf_rec_words(n);
        }
    } else {
        for (int i = threadIdx.x; i < nch * kTileRows; i += blockDim.x) {
            const int c = i >> 4, r = i & 15;
            int32_t base0 = 0, base1 = 0, n_low = 0, n_all = 0;
            for (int rr = 0; rr < kTileRows; ++rr) {
                const int32_t a0 = cnt[2 * (c * 16 + rr)], a1 = cnt[2 * (c * 16 + rr) + 1];
                if (rr < r) { base0 += a0; base1 += a1; }
                n_low += a0;
                n_all += a0 + a1;
            }
            base1 += n_low;
            uint32_t *rec = recs + item_off[(int64_t)blockIdx.x * nch + c];
            if (r == 0) {
                rec[0] = (uint32_t)n_low | ((uint32_t)n_all << 16);
                rec[1] = rec[2] = rec[3] = 0u;
                for (int64_t w = kGgufRecHdrWords + n_all; w < gguf_rec_words(n_all); ++w) rec[w] = 0u;
            }
            const int64_t a = first[i], z = a + cnt[2 * i] + cnt[2 * i + 1];
            for (int64_t k = a; k < z; ++k) {
                const uint32_t col = (uint32_t)cols[k] & 255u, h = (col >> 5) & 1u;
                const int32_t pos = h ? base1++ : base0++;
                rec[kGgufRecHdrWords + pos] = gguf_frag_index((uint32_t)r, col) | (h << 11) | ((uint32_t)bits[k] << 16);
            }
        }
    }
}

static int grid_for(int64_t n, int per) {
    const int64_t g = (n + per - 1) / per;
    return (int)std::min<int64_t>(g, 1 << 30);
}

static bool mode_ok(int m) { return m == BF16X_DTYPE_BF16 || m == BF16X_DTYPE_F32 || m == BF16X_DTYPE_F32_TRUNC; }

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_gguf_quantize(const void *x, int x_dtype, int64_t n, uint8_t *blocks, void *stream) {
    if (n < 0 || n % 32) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_quantize: n must be a multiple of 32");
    if (!mode_ok(x_dtype)) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_quantize: bad x_dtype");
    if (n == 0) return BF16X_OK;
    if (!x || !blocks) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_quantize: null pointer");
    if (reinterpret_cast<uintptr_t>(blocks) & 3u) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_quantize: blocks must be 4-byte aligned");
    const int64_t nb = n / 32;
    gguf_quantize_kernel<<<grid_for(nb, kGCta), kGCta, 0, (cudaStream_t)stream>>>(x, x_dtype, nb, blocks);
    return check_launch("bf16x_gguf_quantize");
}

extern "C" int bf16x_gguf_dequantize(const uint8_t *blocks, int64_t nblocks, void *y, int y_dtype, void *stream) {
    if (nblocks < 0) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_dequantize: bad size");
    if (y_dtype != BF16X_DTYPE_BF16 && y_dtype != BF16X_DTYPE_F32)
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_dequantize: bad y_dtype");
    if (nblocks == 0) return BF16X_OK;
    if (!blocks || !y) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_dequantize: null pointer");
    if (reinterpret_cast<uintptr_t>(blocks) & 3u) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_dequantize: blocks must be 4-byte aligned");
    gguf_dequantize_kernel<<<grid_for(nblocks, kGCta), kGCta, 0, (cudaStream_t)stream>>>(
        blocks, nblocks, y, y_dtype == BF16X_DTYPE_F32);
    return check_launch("bf16x_gguf_dequantize");
}

extern "C" int bf16x_gguf_ovf_count(const void *x, int x_dtype, int64_t rows, int64_t cols, uint32_t *row_off,
                                    void *stream) {
    if (rows < 0 || cols < 0 || cols % 32) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_count: cols must be a multiple of 32");
    if (cols > 65536) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gguf_ovf_count: cols > 65536 (u16 column index)");
    if (!mode_ok(x_dtype)) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_count: bad x_dtype");
    if (!row_off) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_count: null row_off");
    if (rows > 0 && cols > 0 && !x) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_count: null x");
    cudaStream_t st = (cudaStream_t)stream;
    if (rows == 0) {
        const cudaError_t e = cudaMemsetAsync(row_off, 0, 4, st);
        return e == cudaSuccess ? BF16X_OK : set_error(BF16X_ERR_CUDA, "bf16x_gguf_ovf_count: %s", cudaGetErrorString(e));
    }
    gguf_ovf_count_kernel<<<(int)std::min<int64_t>(rows, 65535), 256, 0, st>>>(x, x_dtype, rows, cols, row_off);
    if (int rc = check_launch("bf16x_gguf_ovf_count")) return rc;
    gguf_scan_kernel<<<1, 1024, 0, st>>>(row_off, rows);
    return check_launch("bf16x_gguf_ovf_count scan");
}

extern "C" int bf16x_gguf_ovf_pack(const void *x, int x_dtype, int64_t rows, int64_t cols, const uint32_t *row_off,
                                   uint16_t *ecols, uint16_t *ebits, void *stream) {
    if (rows < 0 || cols < 0 || cols % 32 || cols > 65536) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_pack: bad shape");
    if (!mode_ok(x_dtype)) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_pack: bad x_dtype");
    if (rows == 0 || cols == 0) return BF16X_OK;
    if (!x || !row_off || !ecols || !ebits) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_ovf_pack: null pointer");
    gguf_ovf_pack_kernel<<<(int)std::min<int64_t>(rows, 65535), 256, 0, (cudaStream_t)stream>>>(
        x, x_dtype, rows, cols, row_off, ecols, ebits);
    return check_launch("bf16x_gguf_ovf_pack");
}

extern "C" int bf16x_gguf_apply_ovf(void *y, int y_dtype, int64_t rows, int64_t cols, const uint32_t *row_off,
                                    const uint16_t *ecols, const uint16_t *ebits, int64_t n_entries, void *stream) {
    if (rows < 0 || cols < 0 || n_entries < 0) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_apply_ovf: bad size");
    if (y_dtype != BF16X_DTYPE_BF16 && y_dtype != BF16X_DTYPE_F32)
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_apply_ovf: bad y_dtype");
    if (n_entries == 0) return BF16X_OK;
    if (rows == 0 || !y || !row_off || !ecols || !ebits) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_apply_ovf: null pointer");
    gguf_apply_ovf_kernel<<<grid_for(n_entries, 256), 256, 0, (cudaStream_t)stream>>>(
        y, y_dtype == BF16X_DTYPE_F32, rows, cols, row_off, ecols, ebits, n_entries);
    return check_launch("bf16x_gguf_apply_ovf");
}

static int side_args(const char *who, const uint32_t *row_off, const uint16_t *cols, int64_t rows, int64_t in_f,
                     int64_t n_entries) {
    if (rows < 0 || n_entries < 0) return set_error(BF16X_ERR_INVALID, "%s: bad size", who);
    if (in_f <= 0 || in_f % 256 || in_f > 65536)
        return set_error(BF16X_ERR_UNSUPPORTED, "%s: in_f must be a multiple of 256 and <= 65536", who);
    if (rows > 0 && !row_off) return set_error(BF16X_ERR_INVALID, "%s: null row_off", who);
    if (n_entries > 0 && !cols) return set_error(BF16X_ERR_INVALID, "%s: null columns", who);
    if (n_entries >= (1ll << 30)) return set_error(BF16X_ERR_UNSUPPORTED, "%s: too many entries", who);
    return BF16X_OK;
}

extern "C" int bf16x_gguf_side_index_count(const uint32_t *row_off, const uint16_t *cols, int64_t rows, int64_t in_f,
                                           int64_t n_entries, int32_t *item_off, void *stream) {
    if (int rc = side_args("bf16x_gguf_side_index_count", row_off, cols, rows, in_f, n_entries)) return rc;
    if (!item_off) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_side_index_count: null item_off");
    const int nch = (int)(in_f / 256);
    const int64_t n_tiles = (rows + kTileRows - 1) / kTileRows;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t sh = (size_t)nch * kTileRows * 3 * sizeof(int32_t);
    if (n_tiles > 0) {
        cudaFuncSetAttribute(gguf_side_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh);
        gguf_side_kernel<false><<<(unsigned)n_tiles, 256, sh, st>>>(row_off, cols, nullptr, rows, in_f, n_entries, nch,
                                                                   item_off, nullptr);
        if (int rc = check_launch("bf16x_gguf_side_index_count")) return rc;
    }
    gguf_scan_kernel<<<1, 1024, 0, st>>>(reinterpret_cast<uint32_t *>(item_off), n_tiles * nch);
    return check_launch("bf16x_gguf_side_index_count scan");
}

extern "C" int bf16x_gguf_side_index(const uint32_t *row_off, const uint16_t *cols, const uint16_t *bits, int64_t rows,
                                     int64_t in_f, int64_t n_entries, const int32_t *item_off, uint32_t *item_recs,
                                     void *stream) {
    if (int rc = side_args("bf16x_gguf_side_index", row_off, cols, rows, in_f, n_entries)) return rc;
    if (rows == 0) return BF16X_OK;
    if (!item_off || !item_recs || (n_entries > 0 && !bits))
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_side_index: null pointer");
    const int nch = (int)(in_f / 256);
    const int64_t n_tiles = (rows + kTileRows - 1) / kTileRows;
    const size_t sh = (size_t)nch * kTileRows * 3 * sizeof(int32_t);
    cudaFuncSetAttribute(gguf_side_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sh);
    gguf_side_kernel<true><<<(unsigned)n_tiles, 256, sh, (cudaStream_t)stream>>>(
        row_off, cols, bits, rows, in_f, n_entries, nch, const_cast<int32_t *>(item_off), item_recs);
    return check_launch("bf16x_gguf_side_index");
}
