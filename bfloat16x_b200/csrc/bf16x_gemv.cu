// bf16x_gemv.cu -- fused BF16X decode + GEMV for batch 1..8 (sm_100a).
//
// Replaces _bf16x_gemv_fused_kernel / bf16x_fused_gemv (bf16x_fused.py:32-127)
// and generalises it from batch 1 to batch <= 8.
//
// Design (HBM-bound: the only large stream is the compressed weight):
//   * persistent CTAs, one per SM; a CTA walks tiles of 16 weight rows;
//   * one producer warp streams each tile's compressed rows (368-byte chunks
//     of the resident layout) and the matching activation slice into a ring
//     of shared-memory stages with 1-D bulk copies (the TMA engine), completion
//     counted on mbarriers; consumer warps release stages through a second
//     set of mbarriers;
//   * each consumer warp owns one 256-column chunk per stage; a lane decodes
//     two 32-column groups (rows g and g+8 of the tile) straight into bf16x2
//     registers and feeds them as the A operand of mma.m16n8k16 (rows x k),
//     with the activations as the B operand (k x batch).  The tensor core does
//     the multiply-accumulate, so the CUDA cores only decode: about five
//     integer ops per pair of weights;
//   * at the end of a tile the warps' fp32 partials are summed in a fixed
//     order in shared memory and the exact-delta patches (delta > 7, ~3% of
//     weights) are added as (w_exact - w_saturated) * x by 2*NW lanes per row
//     with a shuffle reduction, so results are deterministic;
//   * every mbarrier wait is bounded (bf16x_common.cuh) and reports a timeout
//     through the device status word instead of hanging.
#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_resident.cuh"
#include "bf16x_status.cuh"

namespace bf16x {

constexpr int kGemvRows = 16;

template <int NW, int BMAX>
struct GemvCfg {
    static constexpr int kPadR = (16 - (NW * kChunkBytes) % 128 + 128) % 128;
    static constexpr int kRowStride = NW * kChunkBytes + kPadR;   // == 16 (mod 128): conflict-free 16-B loads
    static constexpr int kXStride = NW * kChunkElems * 2 + 16;
    static constexpr int kXOff = kGemvRows * kRowStride;
    static constexpr int kStageBytes = (kXOff + BMAX * kXStride + 127) / 128 * 128;
    static constexpr int kStages = (200 * 1024 / kStageBytes) < 8 ? (200 * 1024 / kStageBytes) : 8;
    static constexpr int kRedBytes = NW * kGemvRows * 8 * 4;
    static constexpr int kSmem = kStages * kStageBytes + kRedBytes + 2 * kStages * 8;
    static_assert(kStages >= 2, "stage too large");
};

struct GemvParams {
    const uint8_t *layout;
    const int32_t *patch_off;
    const uint32_t *patches;
    int64_t rows, in_f, row_bytes;
    int nch, n_tiles;
    const uint16_t *x;
    int64_t ldx;
    int batch;
    const uint16_t *bias;
    void *y;
    int y_f32;
    int64_t ldy;
};

__device__ __forceinline__ void mma_bf16_16816(float &c0, float &c1, float &c2, float &c3, uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c0), "+f"(c1), "+f"(c2), "+f"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// mma step J of one group: k-slots (2t, 2t+1 | 2t+8, 2t+9) carry the group's
// columns 4J..4J+3, i.e. pairs 2J (a0/a1) and 2J+1 (a2/a3) for rows g and g+8.
// The B operand of lane (g, t) is x[g][group + 4J .. +3]: one 8-byte load.
template <int J>
__device__ __forceinline__ void group_mma(const uint32_t (&smA)[8], const uint32_t (&dA)[3], uint32_t eAlo,
                                          uint32_t eAhi, const uint32_t (&smB)[8], const uint32_t (&dB)[3],
                                          uint32_t eBlo, uint32_t eBhi, const uint16_t *xq, bool xv, float &c0,
                                          float &c1, float &c2, float &c3) {
    const uint32_t eA = J < 4 ? eAlo : eAhi, eB = J < 4 ? eBlo : eBhi;
    const uint32_t a0 = decode_pair<2 * J>(smA, dA, eA);
    const uint32_t a1 = decode_pair<2 * J>(smB, dB, eB);
    const uint32_t a2 = decode_pair<2 * J + 1>(smA, dA, eA);
    const uint32_t a3 = decode_pair<2 * J + 1>(smB, dB, eB);
    uint2 b = make_uint2(0u, 0u);
    if (xv) b = *reinterpret_cast<const uint2 *>(xq + 4 * J);
    mma_bf16_16816(c0, c1, c2, c3, a0, a1, a2, a3, b.x, b.y);
    if constexpr (J + 1 < 8)
        group_mma<J + 1>(smA, dA, eAlo, eAhi, smB, dB, eBlo, eBhi, xq, xv, c0, c1, c2, c3);
}

__device__ __forceinline__ void chunk_mma(const uint8_t *rowA, const uint8_t *rowB, const uint16_t *xg, bool xv,
                                          int t, float &c0, float &c1, float &c2, float &c3) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int q = 4 * h + t;
        uint32_t smA[8], dA[3], eAlo, eAhi, smB[8], dB[3], eBlo, eBhi;
        load_group(rowA, q, smA, dA, eAlo, eAhi);
        load_group(rowB, q, smB, dB, eBlo, eBhi);
        group_mma<0>(smA, dA, eAlo, eAhi, smB, dB, eBlo, eBhi, xg + 32 * q, xv, c0, c1, c2, c3);
    }
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

template <int NW, int BMAX>
__global__ void __launch_bounds__((NW + 1) * 32, 1) gemv_kernel(const GemvParams p) {
    using C = GemvCfg<NW, BMAX>;
    constexpr int S = C::kStages;
    extern __shared__ __align__(128) uint8_t smem[];
    float *red = reinterpret_cast<float *>(smem + S * C::kStageBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * C::kStageBytes + C::kRedBytes);
    uint64_t *empty = full + S;

    // abort[0]: set by any warp whose bounded wait gave up; abort[1]: the
    // consumers' per-tile decision, read by all of them after a barrier.
    __shared__ volatile int abort_flag[2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        abort_flag[0] = 0;
        abort_flag[1] = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    const int spt = (p.nch + NW - 1) / NW;   // stages per tile
    int slot = 0;
    uint32_t ph = 0;

    if (warp == NW) {
        // ------------------------------------------------------------ producer
        for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const int64_t row0 = (int64_t)tile * kGemvRows;
            const int rv = (int)(p.rows - row0 < kGemvRows ? p.rows - row0 : kGemvRows);
            for (int s = 0; s < spt; ++s) {
                const int c0 = s * NW;
                const int nch = min(NW, p.nch - c0);
                int ok = 1;
                if (lane == 0) ok = !abort_flag[0] && mbar_wait(&empty[slot], ph ^ 1u, &g_status);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) abort_flag[0] = 1;
                    return;
                }
                uint8_t *st = smem + slot * C::kStageBytes;
                if (lane == 0)
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)(rv * nch * kChunkBytes + p.batch * nch * kChunkElems * 2));
                __syncwarp();
                if (lane < rv) {
                    bulk_g2s(st + lane * C::kRowStride,
                             p.layout + (row0 + lane) * p.row_bytes + (int64_t)c0 * kChunkBytes,
                             (uint32_t)(nch * kChunkBytes), &full[slot]);
                } else if (lane >= kGemvRows && lane - kGemvRows < p.batch) {
                    const int b = lane - kGemvRows;
                    bulk_g2s(st + C::kXOff + b * C::kXStride, p.x + b * p.ldx + (int64_t)c0 * kChunkElems,
                             (uint32_t)(nch * kChunkElems * 2), &full[slot]);
                }
                if (++slot == S) { slot = 0; ph ^= 1u; }
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const bool xv = g < p.batch;
    constexpr int TPR = 2 * NW;                 // threads per row in the epilogue
    const int ctid = warp * 32 + lane;
    const int erow = ctid / TPR, esl = ctid % TPR;

    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
        const int64_t row0 = (int64_t)tile * kGemvRows;
        float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
        bool failed = false;
        for (int s = 0; s < spt; ++s) {
            const int nch = min(NW, p.nch - s * NW);
            if (!failed && (abort_flag[0] || !mbar_wait(&full[slot], ph, &g_status))) {
                failed = true;
                abort_flag[0] = 1;
            }
            if (!failed && warp < nch) {
                const uint8_t *st = smem + slot * C::kStageBytes;
                const uint8_t *rowA = st + g * C::kRowStride + warp * kChunkBytes;
                const uint8_t *rowB = rowA + 8 * C::kRowStride;
                const uint16_t *xg = reinterpret_cast<const uint16_t *>(st + C::kXOff + g * C::kXStride) +
                                     warp * kChunkElems;
                chunk_mma(rowA, rowB, xg, xv, t, c0, c1, c2, c3);
            }
            __syncwarp();
            if (lane == 0 && !failed) mbar_arrive(&empty[slot]);
            if (++slot == S) { slot = 0; ph ^= 1u; }
        }

        // ---- epilogue: fixed-order reduction + exact-delta patches
        float *rw = red + warp * kGemvRows * 8;
        rw[g * 8 + 2 * t] = c0;
        rw[g * 8 + 2 * t + 1] = c1;
        rw[(g + 8) * 8 + 2 * t] = c2;
        rw[(g + 8) * 8 + 2 * t + 1] = c3;
        named_bar(1, NW * 32);

        const int64_t grow = row0 + erow;
        float corr[BMAX];
#pragma unroll
        for (int b = 0; b < BMAX; ++b) corr[b] = 0.f;
        if (grow < p.rows) {
            const int32_t lo = __ldg(p.patch_off + grow), hi = __ldg(p.patch_off + grow + 1);
            const uint8_t *lrow = p.layout + grow * p.row_bytes;
            for (int32_t j = lo + esl; j < hi; j += TPR) {
                const uint32_t ent = __ldg(p.patches + j);
                const uint32_t col = ent & 0xFFFFu;
                const uint32_t em = __ldg(lrow + (col >> 8) * kChunkBytes + kEOff + ((col & 255u) >> 4));
                const float dw = bf16_bits_to_f32(patch_bits(ent, em)) - bf16_bits_to_f32(saturated_bits(ent, em));
#pragma unroll
                for (int b = 0; b < BMAX; ++b)
                    if (b < p.batch) corr[b] = fmaf(dw, bf16_bits_to_f32(__ldg(p.x + b * p.ldx + col)), corr[b]);
            }
        }
#pragma unroll
        for (int b = 0; b < BMAX; ++b) {
#pragma unroll
            for (int o = TPR / 2; o; o >>= 1) corr[b] += __shfl_xor_sync(0xffffffffu, corr[b], o);
        }
        if (grow < p.rows && !abort_flag[0]) {
            const float bias = p.bias ? bf16_bits_to_f32(__ldg(p.bias + grow)) : 0.f;
#pragma unroll
            for (int b = 0; b < BMAX; ++b) {
                if (b < p.batch && (b % TPR) == esl) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < NW; ++w) v += red[(w * kGemvRows + erow) * 8 + b];
                    v += corr[b];
                    v += bias;
                    if (p.y_f32)
                        reinterpret_cast<float *>(p.y)[b * p.ldy + grow] = v;
                    else
                        reinterpret_cast<uint16_t *>(p.y)[b * p.ldy + grow] = f32_to_bf16_bits_rn(v);
                }
            }
        }
        if (ctid == 0) abort_flag[1] = abort_flag[0];
        named_bar(1, NW * 32);
        if (abort_flag[1]) return;
    }
}

template <int NW, int BMAX>
static int launch_gemv(const GemvParams &p, cudaStream_t st) {
    using C = GemvCfg<NW, BMAX>;
    int dev = 0;
    cudaGetDevice(&dev);
    static int attr_set[64] = {0};
    static int sms[64] = {0};
    if (dev < 0 || dev >= 64) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv: device index %d", dev);
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<NW, BMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemv: smem attribute: %s", cudaGetErrorString(e));
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        attr_set[dev] = 1;
    }
    const int grid = min(p.n_tiles, max(sms[dev], 1));
    gemv_kernel<NW, BMAX><<<grid, (NW + 1) * 32, C::kSmem, st>>>(p);
    return check_launch("bf16x_gemv");
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int bf16x_gemv(const uint8_t *layout, const int32_t *patch_off, const uint32_t *patches,
                          int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                          const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *stream) {
    if (rows < 0 || in_f <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: bad shape");
    if (in_f > 65536) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv: in_f > 65536");
    if (batch < 1 || batch > 8) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: batch must be 1..8 (got %lld)", (long long)batch);
    if (y_dtype != BF16X_DTYPE_BF16 && y_dtype != BF16X_DTYPE_F32)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: bad y_dtype");
    if (rows == 0) return BF16X_OK;
    if (!layout || !patch_off || !x || !y) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: null pointer");
    const int64_t in_pad = (in_f + kChunkElems - 1) / kChunkElems * kChunkElems;
    if (ldx < in_pad || (ldx % 8) != 0)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: ldx must be a multiple of 8 and >= %lld (zero padded)", (long long)in_pad);
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(layout)) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: x and layout must be 16-byte aligned");
    if (ldy < rows) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: ldy < rows");
    GemvParams p;
    p.layout = layout; p.patch_off = patch_off; p.patches = patches;
    p.rows = rows; p.in_f = in_f; p.row_bytes = resident_row_bytes(in_f);
    p.nch = (int)(in_pad / kChunkElems);
    p.n_tiles = (int)((rows + kGemvRows - 1) / kGemvRows);
    p.x = x; p.ldx = ldx; p.batch = (int)batch;
    p.bias = bias; p.y = y; p.y_f32 = y_dtype == BF16X_DTYPE_F32; p.ldy = ldy;
    cudaStream_t st = (cudaStream_t)stream;
    if (batch == 1) return launch_gemv<4, 1>(p, st);
    if (batch == 2) return launch_gemv<4, 2>(p, st);
    if (batch <= 4) return launch_gemv<4, 4>(p, st);
    return launch_gemv<4, 8>(p, st);
}
