// bf16x_decode.cu -- flat-stream decode with the overflow fix fused in.
//
// Replaces the reference's two-kernel decode (_bf16x_decode_kernel +
// _bf16x_fix_ovf_kernel, bf16x_triton_test.py:11-108) and its host-side
// filter/.item() sync with one pass.  HBM-bound: 1.4375 bytes of streams +
// 5 bytes per overflow entry in, 2 bytes out per weight.
//
//   * Tiles of 8192 consecutive flat elements; each CTA (persistent, up to
//     four per SM) owns a contiguous range of tiles, so its reads and writes
//     walk memory in order and the overflow slice of one tile ends where the
//     next one's begins.
//   * A tile's streams -- 256 sign words, 1792 mantissa words, 768 delta
//     words and 512 emax bytes, every piece 16-byte aligned because the tile
//     is 8192-aligned -- arrive by four bulk copies (TMA engine) into one of
//     three shared-memory stages, the copies of the tile two ahead issued
//     while this one is decoded; a tile that is not whole (the last) or
//     streams that are not 16-byte aligned take plain loads instead.
//   * Thread t decodes group t (32 elements: one sign word, seven mantissa
//     words, three delta words, two emax bytes -- shared-memory strides 7 and
//     3 words touch 32 distinct banks) two elements per step (one funnel
//     shift for both mantissas, one for both deltas, one subtraction for both
//     exponents) and writes four 16-byte chunks into the shared tile, XOR-swizzled so neither these
//     writes nor the linear read-back for the global stores conflict.
//   * The overflow table is sorted, so a tile's entries are the run that
//     starts where the previous tile's ended (one 32-way search per CTA finds
//     the first): the next 512 entries are requested before the tile's
//     streams are waited for, counted below the tile's end with the barrier
//     that publishes the decoded tile, and patch it in shared memory, only
//     where the stream delta is the saturated 7 (the reference decode's rule,
//     opqk_linear.py:367-372).
//   * The tile leaves with coalesced 16-byte stores.
#include <algorithm>
#include <climits>

#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_flat.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

constexpr int kDecThreads = 256;
constexpr int kDecTile = kDecThreads * 32;               // elements per tile
constexpr int kDecSignW = kDecTile / 32;                 // 256 words
constexpr int kDecMantW = kDecTile * 7 / 32;             // 1792 words
constexpr int kDecDeltaW = kDecTile * 3 / 32;            // 768 words
constexpr int kDecEmaxB = kDecTile / 16;                 // 512 bytes
constexpr int kDecStageB = 4 * (kDecSignW + kDecMantW + kDecDeltaW) + kDecEmaxB;   // 11776
constexpr int kDecPrefetch = 2;                          // overflow entries per thread held ahead
constexpr int kDecStages = 3;                            // tiles in flight per CTA: this one + two ahead
constexpr int kDecCtasPerSm = 4;

struct DecStage {
    uint32_t sign[kDecSignW];
    uint32_t mant[kDecMantW];
    uint32_t delta[kDecDeltaW];
    uint8_t emax[kDecEmaxB];
};
static_assert(sizeof(DecStage) == kDecStageB && kDecStageB % 16 == 0, "stage layout");

struct DecSmem {
    DecStage stage[kDecStages];
    uint4 tile[kDecTile / 8];                            // 16 KB of bf16, swizzled 16-byte chunks
    uint64_t bar[kDecStages];
    int64_t slice_lo;                                    // start of the first tile's overflow slice
};

// 16-byte chunk j (0..3) of group t in the swizzled tile: the eight threads of
// a store phase (and the chunks a read phase takes) fall in eight different
// 16-byte bank groups.
__device__ __forceinline__ int dec_chunk(int t, int j) { return 4 * t + (j ^ ((t >> 1) & 3)); }

// Element e (0..8191) of the swizzled tile, as a bf16 index.
__device__ __forceinline__ int dec_elem(int e) {
    const int t = e >> 5, o = e & 31;
    return dec_chunk(t, o >> 3) * 8 + (o & 7);
}

// bf16x2 bits of elements 2P (low half) and 2P+1 (high half) of a group: one
// funnel shift brings both 7-bit mantissas (stream bits 14P..14P+13), one both
// 3-bit deltas (bits 6P..6P+5); both exponents come from one subtraction on
// the two 16-bit halves.  e2 = emax * 0x00010001 + 0x100: the extra 256 in
// the low half keeps (emax - delta) from borrowing out of it, and the mask
// keeps the low 8 bits of each difference, i.e. (emax - delta) & 0xFF.
template <int P>
__device__ __forceinline__ uint32_t decode_flat_pair(uint32_t sw, const uint32_t (&mw)[8], const uint32_t (&dw)[4],
                                                     uint32_t e2) {
    constexpr int MB = 14 * P, DB = 6 * P;
    const uint32_t x = funnel_r(mw[MB >> 5], mw[(MB >> 5) + 1], MB & 31);
    const uint32_t m2 = (x & 0x7Fu) | ((x << 9) & 0x7F0000u);
    const uint32_t y = funnel_r(dw[DB >> 5], dw[(DB >> 5) + 1], DB & 31);
    const uint32_t d2 = (y & 7u) | ((y << 13) & 0x70000u);
    const uint32_t ex = ((e2 - d2) << 7) & 0x7F807F80u;
    const uint32_t s2 = (((sw >> (2 * P)) << 15) & 0x8000u) | ((sw << (30 - 2 * P)) & 0x80000000u);
    return s2 | ex | m2;
}

template <int P>
__device__ __forceinline__ void decode_flat_pairs(uint32_t sw, const uint32_t (&mw)[8], const uint32_t (&dw)[4],
                                                  uint32_t e2a, uint32_t e2b, uint32_t (&pairs)[16]) {
    pairs[P] = decode_flat_pair<P>(sw, mw, dw, P < 8 ? e2a : e2b);
    if constexpr (P + 1 < 16) decode_flat_pairs<P + 1>(sw, mw, dw, e2a, e2b, pairs);
}

// bf16 bits of the 32 elements of one group from its words.
__device__ __forceinline__ void decode_group32(uint32_t sw, const uint32_t (&mw)[8], const uint32_t (&dw)[4],
                                               uint32_t eb0, uint32_t eb1, uint32_t (&pairs)[16]) {
    decode_flat_pairs<0>(sw, mw, dw, eb0 * 0x00010001u + 0x100u, eb1 * 0x00010001u + 0x100u, pairs);
}

__global__ void __launch_bounds__(kDecThreads, kDecCtasPerSm)
flat_decode_kernel(FlatStreams f, uint16_t *__restrict__ out, int64_t n_tiles, int bulk_ok) {
    extern __shared__ __align__(128) uint8_t dec_smem_raw[];
    DecSmem &sm = *reinterpret_cast<DecSmem *>(dec_smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // this CTA's contiguous tiles [tb, te)
    const int64_t tb = n_tiles * blockIdx.x / gridDim.x;
    const int64_t te = n_tiles * (blockIdx.x + 1) / gridDim.x;
    if (tb >= te) return;
    // a tile goes through the bulk copies when it is whole and the streams are aligned
    auto bulk_tile = [&](int64_t t) { return bulk_ok && (t + 1) * kDecTile <= f.n; };
    auto issue = [&](int64_t t, int s) {     // one thread
        DecStage &st = sm.stage[s];
        mbar_arrive_expect_tx(&sm.bar[s], (uint32_t)kDecStageB);
        bulk_g2s(st.sign, f.sign + t * kDecSignW, 4 * kDecSignW, &sm.bar[s]);
        bulk_g2s(st.mant, f.mant + t * kDecMantW, 4 * kDecMantW, &sm.bar[s]);
        bulk_g2s(st.delta, f.delta + t * kDecDeltaW, 4 * kDecDeltaW, &sm.bar[s]);
        bulk_g2s(st.emax, f.emax + t * kDecEmaxB, kDecEmaxB, &sm.bar[s]);
    };
    if (tid == 0)
        for (int s = 0; s < kDecStages; ++s) mbar_init(&sm.bar[s], 1);
    fence_mbar_init();
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kDecStages - 1 && tb + s < te; ++s)
            if (bulk_tile(tb + s)) issue(tb + s, s);

    // start of the first tile's overflow slice; every later tile's slice
    // starts where the previous one ended
    int64_t lo = 0;
    if (f.n_ovf > 0) {
        if (warp == 0) {
            const int64_t r = warp_lower_bound(f.ovf_idx, f.n_ovf, tb * (int64_t)kDecTile);
            if (lane == 0) sm.slice_lo = r;
        }
        __syncthreads();
        lo = sm.slice_lo;
    }

    uint32_t phases = 0u;                                 // bit s: parity of the next phase of stage s
    uint16_t *t16 = reinterpret_cast<uint16_t *>(sm.tile);
    for (int64_t t = tb; t < te; ++t) {
        const int s = (int)((t - tb) % kDecStages);
        const int64_t t0 = t * (int64_t)kDecTile;
        const int64_t t1 = min(t0 + (int64_t)kDecTile, f.n);
        const bool bulk = bulk_tile(t);
        // the tile kDecStages - 1 ahead goes into the stage the previous tile freed
        const int64_t ta = t + kDecStages - 1;
        if (ta < te && tid == 0 && bulk_tile(ta)) issue(ta, (int)((ta - tb) % kDecStages));
        // The next entries of the sorted overflow table, requested before the
        // streams are awaited: those below t1 (a prefix, the table being
        // sorted) are this tile's.
        int32_t e_pos[kDecPrefetch], e_prev[kDecPrefetch];
        uint32_t e_val[kDecPrefetch];
        bool e_in[kDecPrefetch];
#pragma unroll
        for (int k = 0; k < kDecPrefetch; ++k) {
            const int64_t j = lo + tid + (int64_t)k * kDecThreads;
            const bool ok = j < f.n_ovf;
            e_pos[k] = ok ? __ldg(f.ovf_idx + j) : INT32_MAX;
            e_prev[k] = (ok && j > 0) ? __ldg(f.ovf_idx + j - 1) : INT32_MIN;
            e_val[k] = ok ? __ldg(f.ovf_val + j) : 0u;
            e_in[k] = ok && (int64_t)e_pos[k] < t1;
        }

        // ---- base decode of group tid
        const int64_t g = t * kDecThreads + tid;
        if (g * 32 < f.n) {
            uint32_t sw, mw[8], dw[4], eb0, eb1;
            if (bulk) {
                if (!mbar_wait(&sm.bar[s], (phases >> s) & 1u, &g_status)) return;
                const DecStage &st = sm.stage[s];
                sw = st.sign[tid];
#pragma unroll
                for (int i = 0; i < 7; ++i) mw[i] = st.mant[7 * tid + i];
#pragma unroll
                for (int i = 0; i < 3; ++i) dw[i] = st.delta[3 * tid + i];
                eb0 = st.emax[2 * tid];
                eb1 = st.emax[2 * tid + 1];
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
            decode_group32(sw, mw, dw, eb0, eb1, pairs);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                sm.tile[dec_chunk(tid, j)] = make_uint4(pairs[4 * j], pairs[4 * j + 1], pairs[4 * j + 2], pairs[4 * j + 3]);
        }
        if (bulk) phases ^= 1u << s;

        // ---- overflow fix inside shared memory (the counting barriers also
        // publish the decoded tile)
        auto fix = [&](int64_t pos, int64_t prev, uint32_t val) {
            if (prev >= pos) atomicOr(&g_status, kErrOvfUnsorted);
            if (pos < t0) { atomicOr(&g_status, kErrOvfRange); return; }
            const int64_t ei = pos / 16;
            const uint32_t e = bulk ? (uint32_t)sm.stage[s].emax[ei - t0 / 16]
                                    : (ei < f.n_emax ? (uint32_t)__ldg(f.emax + ei) : 0u);
            const int idx = dec_elem((int)(pos - t0));
            const uint32_t cur = t16[idx];
            // the reference substitutes the table delta only where the stream says 7
            if (((cur >> 7) & 0xFFu) == ((e - 7u) & 0xFFu))
                t16[idx] = (uint16_t)((cur & 0x807Fu) | (((e - val) & 0xFFu) << 7));
        };
        int64_t n_in = 0;
        if (f.n_ovf > 0) {
            int full = 1;
#pragma unroll
            for (int k = 0; k < kDecPrefetch; ++k) {
                const int c = __syncthreads_count(e_in[k]);
                n_in += c;
                full &= c == kDecThreads;
            }
#pragma unroll
            for (int k = 0; k < kDecPrefetch; ++k)
                if (e_in[k]) fix(e_pos[k], e_prev[k], e_val[k]);
            // a tile with more entries than were requested ahead (dense
            // overflow): the rest, a block of entries at a time
            for (int64_t j0 = lo + (int64_t)kDecPrefetch * kDecThreads; full; j0 += kDecThreads) {
                const int64_t j = j0 + tid;
                const bool ok = j < f.n_ovf;
                const int64_t pos = ok ? (int64_t)__ldg(f.ovf_idx + j) : INT64_MAX;
                const bool in = ok && pos < t1;
                const int c = __syncthreads_count(in);
                n_in += c;
                full = c == kDecThreads;
                if (in) fix(pos, (int64_t)__ldg(f.ovf_idx + j - 1), __ldg(f.ovf_val + j));
            }
        }
        __syncthreads();

        // ---- coalesced store (linear 16-byte chunks read back through the swizzle)
        const int64_t cnt = t1 - t0;
        if (cnt == kDecTile) {
            uint4 *dst = reinterpret_cast<uint4 *>(out + t0);
#pragma unroll
            for (int i = tid; i < kDecTile / 8; i += kDecThreads) dst[i] = sm.tile[dec_chunk(i >> 2, i & 3)];
        } else {
            for (int64_t i = tid; i < cnt; i += kDecThreads) out[t0 + i] = t16[dec_elem((int)i)];
        }
        lo += n_in;
        __syncthreads();     // the tile and this stage are free
    }
    // entries past every tile (index >= N) or a negative first index
    if (f.n_ovf > 0 && tid == 0) {
        if (te == n_tiles && lo < f.n_ovf) atomicOr(&g_status, kErrOvfRange);
        if (tb == 0 && __ldg(f.ovf_idx) < 0) atomicOr(&g_status, kErrOvfRange);
    }
}

static int decode_grid(int64_t n_tiles) {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return (int)std::min<int64_t>(n_tiles, (int64_t)sms * kDecCtasPerSm);
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
    const int64_t n_tiles = (n + kDecTile - 1) / kDecTile;
    const int bulk_ok = ((reinterpret_cast<uintptr_t>(sign) | reinterpret_cast<uintptr_t>(mant) |
                          reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(emax)) & 15u) == 0;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(flat_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)sizeof(DecSmem));
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_decode: smem attribute: %s", cudaGetErrorString(e));
        attr_set[dev] = true;
    }
    flat_decode_kernel<<<(unsigned)decode_grid(n_tiles), kDecThreads, sizeof(DecSmem), (cudaStream_t)stream>>>(
        f, out, n_tiles, bulk_ok);
    return check_launch("bf16x_decode");
}
