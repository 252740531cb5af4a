// bf16x_repack.cu -- flat dict -> resident layout, and resident -> bf16.
//
// The resident layout (see bf16x_resident.cuh) replaces the per-layer device
// preparation of the reference modules: Bf16xFused.__init__ pads the streams
// and builds a per-row CSR of overflow corrections (bf16x_fused.py:154-192),
// Bf16xGemmLinear.__init__ pads and stages them (bf16x_gemm_fused.py:163-184).
// Here each row is decoded exactly from the flat streams (overflow table
// applied with the reference decode's rule, opqk_linear.py:364-376) and
// re-encoded with row-local 32-column groups and 4-bit deltas, so any in_f
// works (the flat 16-element sub-blocks of the dict may straddle rows when
// in_f % 16 != 0).
//
//   repack_count_kernel : CTA per 16-row tile, record sizes per (tile, chunk)
//   scan_kernel         : exclusive scan of the sizes into ptile_off
//   repack_write_kernel : CTA per 16-row tile, writes chunks and records
#include "bf16x_common.cuh"
#include "bf16x_flat.cuh"
#include "bf16x_resident.cuh"
#include "bf16x_status.cuh"

namespace bf16x {


struct RowSlice {
    int64_t lo, hi;
};

__device__ __forceinline__ RowSlice row_ovf_slice(const FlatStreams &f, int64_t pos0, int64_t in_f) {
    RowSlice s{0, 0};
    if (f.n_ovf > 0) {
        s.lo = warp_lower_bound(f.ovf_idx, f.n_ovf, pos0);
        s.hi = warp_lower_bound(f.ovf_idx, f.n_ovf, pos0 + in_f);
    }
    return s;
}

// Re-encode the 8 columns [c*256 + 8*lane, +8) of one row (lanes 4q..4q+3
// = group q).  Returns the patch mask (bit i = column i needs a patch) and
// fills sm bytes, stored deltas, exact deltas and the group's emax.
struct Enc8 {
    uint32_t sm[8];
    uint32_t d[8];       // exact delta (0..255)
    uint32_t stored[8];  // min(delta, 15)
    uint32_t emax;
    uint32_t pmask;
};

__device__ __forceinline__ Enc8 encode8(const FlatStreams &f, int64_t pos0, int64_t in_f, int c,
                                        const RowSlice &s) {
    const int lane = threadIdx.x & 31;
    Enc8 r;
    uint32_t bits[8];
    uint32_t em = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t k = (int64_t)c * kChunkElems + 8 * lane + i;
        bits[i] = k < in_f ? flat_exact_bits(f, pos0 + k, s.lo, s.hi, 16) : 0u;
        if (k < in_f) em = max(em, (bits[i] >> 7) & 0xFFu);
    }
    em = max(em, __shfl_xor_sync(0xffffffffu, em, 1));   // lanes 4q..4q+3 = group q
    em = max(em, __shfl_xor_sync(0xffffffffu, em, 2));
    r.emax = em;
    r.pmask = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t k = (int64_t)c * kChunkElems + 8 * lane + i;
        if (k < in_f) {
            const uint32_t ex = (bits[i] >> 7) & 0xFFu;
            r.d[i] = em - ex;
            r.sm[i] = ((bits[i] >> 8) & 0x80u) | (bits[i] & 0x7Fu);
            if (r.d[i] > kDeltaSat) r.pmask |= 1u << i;
        } else {
            r.d[i] = min(em, kDeltaSat);   // padding column: finite, multiplied by a zero x
            r.sm[i] = 0u;
        }
        r.stored[i] = min(r.d[i], kDeltaSat);
    }
    return r;
}

// Exclusive scan of a[0..n) in place, a[n] = total (one CTA).
__global__ void __launch_bounds__(1024) scan_kernel(int32_t *a, int64_t n) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t carry_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += 1024) {
        const int64_t i = base + tid;
        const int32_t v = i < n ? a[i] : 0;
        int32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_sums[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int32_t w = warp_sums[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            warp_sums[lane] = w;   // inclusive
        }
        __syncthreads();
        const int32_t carry = carry_s;
        const int32_t excl = carry + (warp ? warp_sums[warp - 1] : 0) + x - v;
        if (i < n) a[i] = excl;
        __syncthreads();
        if (tid == 1023) carry_s = excl + v;
        __syncthreads();
    }
    if (tid == 0) a[n] = carry_s;
}

// One CTA per 16-row tile, one warp per row.  Counts the patches (exact delta
// > 15) of every (tile, chunk) and writes the record sizes in words.
__global__ void __launch_bounds__(kTileRows * 32)
repack_count_kernel(FlatStreams f, int64_t in_f, int64_t row0, int64_t row1, int nch, int32_t *rec_sizes) {
    extern __shared__ int cnt[];   // [nch]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int c = threadIdx.x; c < nch; c += blockDim.x) cnt[c] = 0;
    __syncthreads();
    const int64_t r = row0 + (int64_t)blockIdx.x * kTileRows + warp;
    if (r < row1) {
        const int64_t pos0 = r * in_f;
        const RowSlice s = row_ovf_slice(f, pos0, in_f);
        for (int c = 0; c < nch; ++c) {
            const Enc8 e = encode8(f, pos0, in_f, c, s);
            int n = __popc(e.pmask);
#pragma unroll
            for (int o = 16; o; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
            if (lane == 0 && n) atomicAdd(&cnt[c], n);
        }
    }
    __syncthreads();
    for (int c = threadIdx.x; c < nch; c += blockDim.x)
        rec_sizes[(int64_t)blockIdx.x * nch + c] = (int32_t)rec_words(cnt[c]);
}

// One CTA per 16-row tile: pass A counts each row's patches per chunk and
// quarter (64-column block), pass B writes the resident chunks, the records'
// emax bytes and headers, and the entries sorted by (quarter, row, column).
__global__ void __launch_bounds__(kTileRows * 32)
repack_write_kernel(FlatStreams f, int64_t in_f, int64_t row0, int64_t row1, int nch,
                    const int32_t *__restrict__ ptile_off, uint8_t *__restrict__ layout,
                    uint32_t *__restrict__ precs) {
    extern __shared__ uint16_t rc[];   // [16][nch][4]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tile = blockIdx.x;
    const int64_t r = row0 + tile * kTileRows + warp;
    const bool valid = r < row1;
    const int64_t pos0 = r * in_f;
    const RowSlice s = valid ? row_ovf_slice(f, pos0, in_f) : RowSlice{0, 0};
    const int quarter = lane >> 3;     // lanes 8q..8q+7: columns 64q..64q+63
    for (int c = 0; c < nch; ++c) {
        int n = 0;
        if (valid) {
            const Enc8 e = encode8(f, pos0, in_f, c, s);
            n = __popc(e.pmask);
#pragma unroll
            for (int o = 4; o; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);   // sum within the quarter
        }
        if ((lane & 7) == 0) rc[(warp * nch + c) * 4 + quarter] = (uint16_t)n;
    }
    __syncthreads();
    const int64_t row_bytes = resident_row_bytes(in_f);
    uint8_t *row = layout + (r - row0) * row_bytes;
    for (int c = 0; c < nch; ++c) {
        int qtot[4] = {0, 0, 0, 0}, qstart[4] = {0, 0, 0, 0};
        for (int q = 0; q < kTileRows; ++q) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int v = rc[(q * nch + c) * 4 + k];
                if (q < warp) qstart[k] += v;
                qtot[k] += v;
            }
        }
        const int n_q0 = qtot[0], n_low = qtot[0] + qtot[1], n_q012 = n_low + qtot[2], n_all = n_q012 + qtot[3];
        uint32_t *rec = precs + ptile_off[tile * nch + c];
        if (warp == 0 && lane == 0) {
            rec[kRecHdr] = (uint32_t)n_low | ((uint32_t)n_all << 16);
            rec[kRecHdr + 1] = (uint32_t)n_q0 | ((uint32_t)n_q012 << 16);
        }
        if (warp == kTileRows - 1) {
            const int64_t used = kRecHdrWords + n_all, words = rec_words(n_all);
            for (int64_t w = used + lane; w < words; w += 32) rec[w] = 0u;
        }
        if (!valid) {
            if (lane < 2) rec[2 * warp + lane] = 0u;   // emax of a row past the end
            continue;
        }
        const Enc8 e = encode8(f, pos0, in_f, c, s);
        uint8_t *chunk = row + (int64_t)c * kChunkBytes;
        uint2 smv;
        smv.x = e.sm[0] | (e.sm[1] << 8) | (e.sm[2] << 16) | (e.sm[3] << 24);
        smv.y = e.sm[4] | (e.sm[5] << 8) | (e.sm[6] << 16) | (e.sm[7] << 24);
        *reinterpret_cast<uint2 *>(chunk + kSmOff + 8 * lane) = smv;
        // the lane's 8 columns are pairs 4(lane&3)..+3 of group lane>>2: one
        // delta word, at slot pp for its pair pp
        uint32_t dword = 0;
#pragma unroll
        for (int pp = 0; pp < 4; ++pp)
            dword |= (e.stored[2 * pp] << (4 * pp)) | (e.stored[2 * pp + 1] << (16 + 4 * pp));
        *reinterpret_cast<uint32_t *>(chunk + kDOff + 4 * lane) = dword;
        if ((lane & 3) == 0) reinterpret_cast<uint8_t *>(rec)[8 * warp + (lane >> 2)] = (uint8_t)e.emax;
        // ordered entries: exclusive prefix of the per-lane counts within the quarter
        const int n = __popc(e.pmask);
        int x = n;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if ((lane & 7) >= o) x += y;
        }
        const int qbase = quarter == 0 ? 0 : quarter == 1 ? n_q0 : quarter == 2 ? n_low : n_q012;
        uint32_t *dst = rec + kRecHdrWords + qbase + qstart[quarter] + (x - n);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (e.pmask & (1u << i)) {
                const uint32_t col = (uint32_t)(8 * lane + i);
                const uint32_t bits = ((e.sm[i] & 0x80u) << 8) | (((e.emax - e.d[i]) & 0xFFu) << 7) | (e.sm[i] & 0x7Fu);
                *dst++ = frag_index((uint32_t)warp, col) | ((col >> 7) << 11) | (bits << 16);
            }
        }
    }
}

// Checks that the overflow index is strictly ascending inside [0, n).
__global__ void validate_ovf_kernel(const int32_t *idx, int64_t n_ovf, int64_t n) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n_ovf;
         j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t v = idx[j];
        if (v < 0 || v >= n) atomicOr(&g_status, kErrOvfRange);
        if (j > 0 && (int64_t)idx[j - 1] >= v) atomicOr(&g_status, kErrOvfUnsorted);
    }
}

// Resident layout -> bf16 bits.  One CTA per 16-row tile: warp w decodes row
// w (lane = one 32-column group, lanes 8u..8u+7 cover chunk 4*it + u, emax
// from the chunk's record), then the CTA applies the tile's patch entries.
__global__ void __launch_bounds__(kTileRows * 32)
resident_decode_kernel(const uint8_t *__restrict__ layout, const int32_t *__restrict__ ptile_off,
                       const uint32_t *__restrict__ precs, int64_t rows, int64_t in_f,
                       uint16_t *__restrict__ out, int64_t ld_out, bool vec_ok) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tile = blockIdx.x;
    const int64_t r = tile * kTileRows + warp;
    const int64_t row_bytes = resident_row_bytes(in_f);
    const int nch = (int)((in_f + kChunkElems - 1) / kChunkElems);
    if (r < rows) {
        const uint8_t *row = layout + r * row_bytes;
        uint16_t *orow = out + r * ld_out;
        for (int c = lane >> 3; c < nch; c += 4) {
            const int q = lane & 7;
            uint32_t sm[8], dw[4];
            load_group(row + (int64_t)c * kChunkBytes, q, sm, dw);
            const uint32_t e2 = emax_x2(rec_emax(precs + ptile_off[tile * nch + c], warp, q));
            GroupPairs g;
            decode_pairs_from<0>(g, sm, dw, e2);
            const int64_t k0 = (int64_t)c * kChunkElems + 32 * q;
            if (k0 + 32 <= in_f && vec_ok) {
                uint4 *dst = reinterpret_cast<uint4 *>(orow + k0);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    dst[i] = make_uint4(g.w[4 * i], g.w[4 * i + 1], g.w[4 * i + 2], g.w[4 * i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (k0 + i < in_f) orow[k0 + i] = (uint16_t)(g.w[i >> 1] >> (16 * (i & 1)));
            }
        }
    }
    __syncthreads();
    for (int c = 0; c < nch; ++c) {
        const uint32_t *rec = precs + ptile_off[tile * nch + c];
        const int n_all = (int)(rec[kRecHdr] >> 16);
        for (int j = threadIdx.x; j < n_all; j += blockDim.x) {
            const uint32_t ent = rec[kRecHdrWords + j];
            uint32_t rt, cc;
            frag_position(ent, rt, cc);
            out[(tile * kTileRows + rt) * ld_out + (int64_t)c * kChunkElems + cc] = (uint16_t)(ent >> 16);
        }
    }
}

static int check_flat_args(const char *who, const uint32_t *sign, int64_t ns, const uint32_t *mant, int64_t nm,
                           const uint32_t *delta, int64_t nd, const uint8_t *emax, int64_t ne,
                           const int32_t *oi, const uint8_t *ov, int64_t no, int64_t out_f, int64_t in_f,
                           int64_t row0, int64_t row1) {
    if (out_f < 0 || in_f <= 0) return set_error(BF16X_ERR_INVALID, "%s: bad shape", who);
    if (in_f > 65536) return set_error(BF16X_ERR_UNSUPPORTED, "%s: in_f > 65536 is not supported by the resident layout", who);
    if (row0 < 0 || row1 < row0 || row1 > out_f) return set_error(BF16X_ERR_INVALID, "%s: bad row range", who);
    const int64_t n = out_f * in_f;
    if (n > 0 && (!sign || !mant || !delta || !emax)) return set_error(BF16X_ERR_INVALID, "%s: null stream", who);
    if (ns < (n + 31) / 32 || nm < (7 * n + 31) / 32 || nd < (3 * n + 31) / 32 || ne < (n + 15) / 16)
        return set_error(BF16X_ERR_INVALID, "%s: stream shorter than out_f*in_f elements need", who);
    if (no < 0 || (no > 0 && (!oi || !ov))) return set_error(BF16X_ERR_INVALID, "%s: bad overflow table", who);
    return BF16X_OK;
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int64_t bf16x_resident_row_bytes(int64_t in_f) { return in_f > 0 ? resident_row_bytes(in_f) : 0; }

extern "C" int bf16x_repack_count(const uint32_t *sign, int64_t n_sign_words,
                                  const uint32_t *mant, int64_t n_mant_words,
                                  const uint32_t *delta, int64_t n_delta_words,
                                  const uint8_t *emax, int64_t n_emax,
                                  const int32_t *ovf_idx, const uint8_t *ovf_val, int64_t n_ovf,
                                  int64_t out_f, int64_t in_f, int64_t row0, int64_t row1,
                                  int32_t *ptile_off, void *stream) {
    int rc = check_flat_args("bf16x_repack_count", sign, n_sign_words, mant, n_mant_words, delta, n_delta_words,
                             emax, n_emax, ovf_idx, ovf_val, n_ovf, out_f, in_f, row0, row1);
    if (rc) return rc;
    if (!ptile_off) return set_error(BF16X_ERR_INVALID, "bf16x_repack_count: null ptile_off");
    cudaStream_t st = (cudaStream_t)stream;
    FlatStreams f{sign, n_sign_words, mant, n_mant_words, delta, n_delta_words,
                  emax, n_emax, ovf_idx, ovf_val, n_ovf, out_f * in_f};
    const int64_t rows = row1 - row0;
    const int nch = (int)((in_f + kChunkElems - 1) / kChunkElems);
    const int64_t n_tiles = (rows + kTileRows - 1) / kTileRows;
    if (n_ovf > 0) {
        validate_ovf_kernel<<<(unsigned)std::min<int64_t>((n_ovf + 255) / 256, 4096), 256, 0, st>>>(ovf_idx, n_ovf, f.n);
        if ((rc = check_launch("validate_ovf_kernel"))) return rc;
    }
    if (n_tiles > 0) {
        repack_count_kernel<<<(unsigned)n_tiles, kTileRows * 32, nch * sizeof(int), st>>>(
            f, in_f, row0, row1, nch, ptile_off);
        if ((rc = check_launch("repack_count_kernel"))) return rc;
    }
    scan_kernel<<<1, 1024, 0, st>>>(ptile_off, n_tiles * nch);
    return check_launch("scan_kernel");
}

extern "C" int bf16x_repack(const uint32_t *sign, int64_t n_sign_words,
                            const uint32_t *mant, int64_t n_mant_words,
                            const uint32_t *delta, int64_t n_delta_words,
                            const uint8_t *emax, int64_t n_emax,
                            const int32_t *ovf_idx, const uint8_t *ovf_val, int64_t n_ovf,
                            int64_t out_f, int64_t in_f, int64_t row0, int64_t row1,
                            const int32_t *ptile_off, uint8_t *layout, uint32_t *precs,
                            void *stream) {
    int rc = check_flat_args("bf16x_repack", sign, n_sign_words, mant, n_mant_words, delta, n_delta_words,
                             emax, n_emax, ovf_idx, ovf_val, n_ovf, out_f, in_f, row0, row1);
    if (rc) return rc;
    if (!ptile_off || !layout || !precs) return set_error(BF16X_ERR_INVALID, "bf16x_repack: null output");
    if ((reinterpret_cast<uintptr_t>(layout) | reinterpret_cast<uintptr_t>(precs)) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_repack: layout and records must be 16-byte aligned");
    const int64_t rows = row1 - row0;
    if (rows == 0) return BF16X_OK;
    FlatStreams f{sign, n_sign_words, mant, n_mant_words, delta, n_delta_words,
                  emax, n_emax, ovf_idx, ovf_val, n_ovf, out_f * in_f};
    const int nch = (int)((in_f + kChunkElems - 1) / kChunkElems);
    const int64_t n_tiles = (rows + kTileRows - 1) / kTileRows;
    repack_write_kernel<<<(unsigned)n_tiles, kTileRows * 32, 4 * kTileRows * nch * sizeof(uint16_t),
                          (cudaStream_t)stream>>>(f, in_f, row0, row1, nch, ptile_off, layout, precs);
    return check_launch("repack_write_kernel");
}

extern "C" int bf16x_resident_decode(const uint8_t *layout, const int32_t *ptile_off,
                                     const uint32_t *precs, int64_t rows, int64_t in_f,
                                     uint16_t *out, int64_t ld_out, void *stream) {
    if (rows < 0 || in_f <= 0 || ld_out < in_f)
        return set_error(BF16X_ERR_INVALID, "bf16x_resident_decode: bad shape");
    if (rows == 0) return BF16X_OK;
    if (!layout || !ptile_off || !precs || !out)
        return set_error(BF16X_ERR_INVALID, "bf16x_resident_decode: null pointer");
    if (reinterpret_cast<uintptr_t>(layout) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_resident_decode: layout must be 16-byte aligned");
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) && (ld_out % 8 == 0);
    resident_decode_kernel<<<(unsigned)((rows + kTileRows - 1) / kTileRows), kTileRows * 32, 0,
                             (cudaStream_t)stream>>>(layout, ptile_off, precs, rows, in_f, out, ld_out, vec_ok);
    return check_launch("resident_decode_kernel");
}
