// bf16x_flat.cuh -- device helpers that read the flat BF16X streams of the
// bf16x_quantize dict (opqk_linear.py:291-324): LSB-first int32 bit streams,
// element i's b-bit field at bits [i*b, i*b+b) of the stream.
#pragma once

#include "bf16x_common.cuh"

namespace bf16x {

struct FlatStreams {
    const uint32_t *sign;  int64_t n_sign;
    const uint32_t *mant;  int64_t n_mant;
    const uint32_t *delta; int64_t n_delta;
    const uint8_t *emax;   int64_t n_emax;
    const int32_t *ovf_idx;
    const uint8_t *ovf_val;
    int64_t n_ovf;
    int64_t n;             // out_f * in_f
};

__device__ __forceinline__ uint32_t ld_word(const uint32_t *w, int64_t nw, int64_t i) {
    return (i >= 0 && i < nw) ? __ldg(w + i) : 0u;
}

// b-bit field of element i (b <= 8); words past nw read as zero.
__device__ __forceinline__ uint32_t flat_field(const uint32_t *w, int64_t nw, int64_t i, int b) {
    const int64_t bit = i * b;
    const int64_t wi = bit >> 5;
    const uint32_t sh = (uint32_t)(bit & 31);
    const uint32_t lo = ld_word(w, nw, wi);
    const uint32_t hi = (sh + b > 32) ? ld_word(w, nw, wi + 1) : 0u;
    return funnel_r(lo, hi, sh) & ((1u << b) - 1u);
}

// Leftmost index j in [lo, hi) with idx[j] >= key (idx ascending), else hi.
__device__ __forceinline__ int64_t lower_bound_dev(const int32_t *idx, int64_t lo, int64_t hi, int64_t key) {
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((int64_t)__ldg(idx + mid) < key) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// Warp-cooperative lower_bound over the whole ascending table: 32 probes per
// round narrow the range 33-fold.  Every lane returns the same result.
__device__ __forceinline__ int64_t warp_lower_bound(const int32_t *idx, int64_t n, int64_t key) {
    const int lane = threadIdx.x & 31;
    int64_t lo = 0, hi = n;            // answer in [lo, hi]
    while (hi - lo > 32) {
        const int64_t span = hi - lo;
        const int64_t probe = lo + (span * (lane + 1)) / 33;   // strictly inside [lo, hi)
        const bool less = (int64_t)__ldg(idx + probe) < key;
        const unsigned m = __ballot_sync(0xffffffffu, less);
        // probes are increasing in lane; the ones with idx < key form a prefix
        const int cnt = __popc(m);
        const int64_t new_lo = cnt ? lo + (span * cnt) / 33 + 1 : lo;
        const int64_t new_hi = cnt < 32 ? lo + (span * (cnt + 1)) / 33 : hi;
        lo = new_lo;
        hi = new_hi;
    }
    // final linear step over at most 32 candidates
    const int64_t j = lo + lane;
    const bool less = j < hi && (int64_t)__ldg(idx + j) < key;
    const unsigned m = __ballot_sync(0xffffffffu, less);
    return lo + __popc(m);
}

// Exact bf16 bits of flat element pos: a saturated stream delta (7) takes the
// true delta of the table entry AT pos, and stays 7 when the table has none.
// For the complete tables bf16x_quantize writes (every stream 7 listed) this
// is the reference decode (opqk_linear.py:364-376, whose searchsorted always
// lands on pos); for the filtered tables of the reference's GPU paths (only
// delta > 7 kept, bf16x_triton_test.py:96, bf16x_fused.py:168-170) it is their
// exact-position fix.  The row's slice [lo, hi) of the table is searched.
// exponent = (emax - d) & 0xFF.
__device__ __forceinline__ uint32_t flat_exact_bits(const FlatStreams &f, int64_t pos,
                                                    int64_t lo, int64_t hi, int sub) {
    const uint32_t m = flat_field(f.mant, f.n_mant, pos, 7);
    uint32_t d = flat_field(f.delta, f.n_delta, pos, 3);
    const uint32_t s = flat_field(f.sign, f.n_sign, pos, 1);
    if (d == 7u && hi > lo) {
        const int64_t loc = lower_bound_dev(f.ovf_idx, lo, hi, pos);
        if (loc < hi && (int64_t)__ldg(f.ovf_idx + loc) == pos) d = __ldg(f.ovf_val + loc);
    }
    const int64_t ei = pos / sub;
    const uint32_t e = ei < f.n_emax ? __ldg(f.emax + ei) : 0u;
    return (s << 15) | (((e - d) & 0xFFu) << 7) | m;
}

}  // namespace bf16x
