// bf16x_gemv.cu -- fused BF16X decode + GEMV for batch 1..16 (sm_100a).
//
// Replaces _bf16x_gemv_fused_kernel / bf16x_fused_gemv (bf16x_fused.py:32-127)
// and generalises it from batch 1 to batch <= 16 (above 8 each decoded
// fragment feeds two mma, one per group of 8 activation rows).
//
// Design (HBM-bound: the only large stream is the compressed weight):
//   * work items are (16-row tile, 256-column chunk) pairs in tile-major
//     order; persistent CTAs (8 to 12 warps per SM) split them stream-K style,
//     every warp a contiguous, equal range, so every SM streams the same
//     number of bytes whatever the shape;
//   * each warp feeds itself: a ring of shared-memory slots filled by the
//     TMA engine -- 16 weight rows x 384 bytes (128-byte swizzled), the
//     activation slice, and the (tile, chunk) patch record with the groups'
//     emax -- completion counted on one mbarrier per slot; a slot is refilled
//     right after it is consumed, so S items per warp are always in flight
//     and no warp waits for another;
//   * a lane decodes two 32-column groups (rows g and g+8) straight into the
//     A fragments of mma.m16n8k16 (about five integer ops per pair of
//     weights) and multiplies them with the activations as the B operand
//     (k x batch): the tensor core does the multiply-accumulate.  The rare
//     weights whose exponent is more than 15 below their group's largest
//     enter the products saturated (exponent emax - 15); their record
//     entries then add (exact - saturated) * x to correction sums of their
//     rows, so the sum is that of the exact weights.  Items with many
//     entries (exact zeros, say) instead pass their fragments through the
//     consumed weight slot, where the exact values are stored over them;
//   * a tile split between warps is finished by whichever warp arrives last
//     (an atomic counter per tile in the workspace), summing the pieces in a
//     fixed order, so results are deterministic and no warp ever waits;
//   * launched with programmatic stream serialization: the next GEMV of a
//     stream (the next layer) starts on the SMs this one frees and requests
//     its weights before it waits for this kernel to complete;
//   * every mbarrier wait is bounded (bf16x_common.cuh) and reports a timeout
//     through the device status word instead of hanging.
#include <algorithm>
#include <type_traits>
#include <mutex>

#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_gguf.cuh"
#include "bf16x_resident.cuh"
#include "bf16x_status.cuh"
#include "bf16x_tmap.h"
#include "bf16x_wait.cuh"

namespace bf16x {

constexpr int kMaxRanks = 8;          // GPUs of one NVSwitch domain reached by the collective epilogue
constexpr int kPcapWords = 256;      // record words staged per slot: emax, header, 222 entries (more: from L2)
constexpr int kSparseEntries = 8;    // items with more patch entries take the fragment round trip
constexpr int kXRowBytes = kChunkElems * 2;

// Configuration per (batch bound, warps per CTA).  Shared memory holds the
// weight slots of all warps first (16 rows x 384 bytes each, 1024-byte
// aligned for the 128-byte swizzle), then every warp's activation + record
// slots, zeros, record offsets and mbarriers.  12-warp configurations get
// 2-slot rings, 8-warp ones 3-slot rings (see warps_for); 9..16 rows with the
// activation block 1-slot rings.
//
// XRES (5..16 activation rows, in_f <= 4096): the whole activation block is
// copied once per CTA into shared memory and every item reads its chunk
// there, instead of copying a 4 KB slice into its slot; with records staged
// to 160 words (126 entries) the slots then shrink enough for 12 warps per SM.
constexpr int kXResChunks = 16;      // in_f <= 4096
//
// FMT selects the weight format: kFmtResident (the resident layout) or
// kFmtGguf (GGUF blocks in place, bf16x_gguf.cuh: 16 rows x 368 bytes per
// item, no swizzle, records of side-table entries only).
constexpr int kFmtResident = 0;
constexpr int kFmtGguf = 1;

template <int BMAX, int NW, bool XRES = false, int FMT = kFmtResident>
struct GemvCfg {
    static constexpr bool kGguf = FMT == kFmtGguf;
    static constexpr int kWBytes = kGguf ? kTileRows * kGgufChunkBytes : kTileRows * kChunkBytes;  // 5888 / 6144
    static constexpr int kRecHdrW = kGguf ? kGgufRecHdrWords : kRecHdrWords;   // words before the entries
    static constexpr int kPOff = XRES ? 0 : BMAX * kXRowBytes;              // record after the activations
    static constexpr int kPcap = XRES ? 160 : kGguf ? 128 : kPcapWords;   // XRES: 126 entries staged, GGUF: 124
    static constexpr int kXRSlot = kPOff + kPcap * 4;
    static constexpr int kPerSlot = kWBytes + kXRSlot;
    static constexpr int kXCache = XRES ? kXResChunks * BMAX * kXRowBytes : 0;
    // NW = 6: two CTAs per SM (half the shared memory each), see warps_for
    static constexpr int kCtasPerSm = NW == 6 ? 2 : 1;
    static constexpr int kBudget = (kCtasPerSm == 2 ? 110 * 1024 : 224 * 1024) - kXCache;   // slots
    // 9..16 rows with the CTA's activation block: one slot per warp, so that
    // 12 warps fit beside the 128 KB block (more warps in flight beat
    // deeper rings here: 128256x4096 0.203 -> 0.188 ms)
    static constexpr int kMinStages = (BMAX > 8 && XRES) ? 1 : 2;
    static constexpr int kWarpsFit = kBudget / (kMinStages * kPerSlot);
    static constexpr int kWarps = NW < kWarpsFit ? NW : kWarpsFit;
    static constexpr int kStagesFit = kBudget / kWarps / kPerSlot;
    static constexpr int kStages = kStagesFit < 3 ? kStagesFit : 3;
    static constexpr int kWOff = 0;                                          // [warp][stage] weight rows
    static constexpr int kXROff = kWarps * kStages * kWBytes;                // [warp][stage] x + record
    static constexpr int kXCOff = kXROff + kWarps * kStages * kXRSlot;       // [chunk][BMAX][256] (XRES)
    static constexpr int kZeroOff = kXCOff + kXCache;                        // 512 zero bytes
    static constexpr int kRecOff = kZeroOff + 512;                           // per slot record offset
    static constexpr int kBarOff = kRecOff + kWarps * kStages * 8;
    static constexpr int kCtaOff = kBarOff + kWarps * kStages * 8 + 8;       // after the x barrier: finished warps
    static constexpr int kSmem = kCtaOff + 16 + 1024;                        // + base alignment
    static_assert(kStages >= kMinStages, "ring too shallow for this configuration");
    static_assert(kCtasPerSm == 1 || 2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM must fit");
    static_assert(kWBytes % (kGguf ? 128 : 1024) == 0 && kXRSlot % 128 == 0 && kPOff % 16 == 0 &&
                      kXCOff % 128 == 0, "slot alignment");
    static_assert(!(kGguf && XRES), "the GGUF form stages its activations per item");
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct GemvParams {
    CUtensorMap wmap;   // resident layout [rows][chunks][3 lines], box 16 rows x 1 chunk, 128B swizzle;
                        // GGUF: blocks as [rows][row_bytes / 4] u32, box 16 rows x 92 words
    CUtensorMap xmap;   // activations [batch][in_pad] bf16, box BMAX rows x 256 columns
    const uint8_t *layout;
    const int32_t *ptile_off;
    const uint32_t *precs;
    int64_t rows, row_bytes;
    int has_rec;        // GGUF: side-table records given (the resident layout always has records)
    int nch, n_tiles;
    int64_t T;          // items = n_tiles * nch
    int64_t W;          // warps taking part in the partition (<= T)
    const uint16_t *x;
    int64_t ldx;
    int batch;
    const uint16_t *bias;
    void *y;
    int y_f32;
    int64_t ldy;
    int32_t *tile_cnt;  // n_tiles counters, zero between launches
    float *partials;    // scratch: W x 2 x [16][8]
    // Collective epilogue (bf16x_gemv_peers, nranks > 1).  Every output is
    // sent as one 64-bit word (fp32 bits | launch epoch << 32) to ll[q] of
    // every rank q: mode 0 (gather) at [b][row0 + row] -- this rank's rows of
    // the whole [batch][out_total] output; mode 1 (reduce) at
    // [rank][b][row] -- this rank's partial sums of all out_total rows.  Each
    // GPU then waits for the words of its own ll[rank] that carry this
    // launch's epoch and writes y from them (mode 1: the sum over ranks, in
    // rank order).  state: this GPU's [finished CTAs, epoch of the last launch].
    int nranks, rank, mode;
    uint64_t *ll[kMaxRanks];
    int64_t ll_ld, out_total, row0;
    uint32_t *state;
};

__device__ __forceinline__ void mma_bf16_16816(float &c0, float &c1, float &c2, float &c3, uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c0), "+f"(c1), "+f"(c2), "+f"(c3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Decode step J of one group pair: k-slots (2t, 2t+1 | 2t+8, 2t+9) of mma
// step J carry the group's columns 4J..4J+3, i.e. pairs 2J (a0/a1) and 2J+1
// (a2/a3) of rows g (a0/a2) and g+8 (a1/a3).
struct StepFrag {
    uint32_t a0, a1, a2, a3;
};

template <int J>
__device__ __forceinline__ StepFrag decode_step(const uint32_t (&smA)[8], const uint32_t (&dA)[4], uint32_t eA,
                                                const uint32_t (&smB)[8], const uint32_t (&dB)[4], uint32_t eB) {
    return StepFrag{decode_pair<2 * J>(smA, dA, eA), decode_pair<2 * J>(smB, dB, eB),
                    decode_pair<2 * J + 1>(smA, dA, eA), decode_pair<2 * J + 1>(smB, dB, eB)};
}

// 16-byte shared-memory load by the lanes whose predicate is set; the others
// get zeros without touching shared memory (no wavefront for them).
__device__ __forceinline__ uint4 lds128_if(const void *ptr, bool pred) {
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t@q ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n\t}"
                 : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w) : "r"(smem_u32(ptr)), "r"((int)pred) : "memory");
    return v;
}

// The patch entries of the item: the first cap - kRecHdrWords are
// staged in shared memory with the record, later ones are read from the
// record in global memory (precs + *rof).
struct ItemPatches {
    const uint32_t *rec;
    const uint32_t *precs;
    const int64_t *rof;
    int cap;                                  // record words staged in shared memory
    int hdr;                                  // record words before the first entry
    __device__ __forceinline__ uint32_t entry(int j) const {
        return hdr + j < cap ? rec[hdr + j] : __ldg(precs + *rof + hdr + j);
    }
};

// (exact - saturated) value of a patched weight: its products go in with the
// saturated decode (exponent emax - 15, same sign and mantissa).
__device__ __forceinline__ float patch_delta(uint32_t ent, uint32_t emax) {
    const uint32_t ex = ent >> 16;
    const uint32_t sat = (ex & 0x807Fu) | (((emax - kDeltaSat) & 0xFFu) << 7);
    return bf16_bits_to_f32(ex) - bf16_bits_to_f32(sat);
}

// Correction of one patched weight (row rr, column cc of the item; dv = 0
// when there is none), taken by the four lanes with g = rr % 8: dv * x[b][cc]
// for the lane's batch columns b = 2t, 2t+1 (and 8+2t, 8+2t+1 when BMAX > 8)
// into the correction sums pc / pd, laid out like the mma accumulators
// (registers 0/1 row g, 2/3 row g + 8).  No branches: the other lanes add 0.
template <int BMAX>
__device__ __forceinline__ void add_patch(uint32_t key, float dv, bool on, int g, int t, const uint16_t *xs,
                                          float (&pc)[4], float (&pd)[4]) {
    const uint32_t rr = key >> 8, cc = key & 0xFFu;
    const bool mine = on && (int)(rr & 7u) == g;
    const float w = mine ? dv : 0.f;
    const bool top = rr < 8;
    const int b0 = 2 * t;
    const float x0 = b0 < BMAX ? bf16_bits_to_f32(xs[b0 * kChunkElems + cc]) : 0.f;
    const float x1 = b0 + 1 < BMAX ? bf16_bits_to_f32(xs[(b0 + 1) * kChunkElems + cc]) : 0.f;
    const float v0 = mine ? w * x0 : 0.f, v1 = mine ? w * x1 : 0.f;
    pc[0] += top ? v0 : 0.f;
    pc[1] += top ? v1 : 0.f;
    pc[2] += top ? 0.f : v0;
    pc[3] += top ? 0.f : v1;
    if constexpr (BMAX > 8) {
        const float v2 = mine ? w * bf16_bits_to_f32(xs[(8 + b0) * kChunkElems + cc]) : 0.f;
        const float v3 = mine ? w * bf16_bits_to_f32(xs[(9 + b0) * kChunkElems + cc]) : 0.f;
        pd[0] += top ? v2 : 0.f;
        pd[1] += top ? v3 : 0.f;
        pd[2] += top ? 0.f : v2;
        pd[3] += top ? 0.f : v3;
    }
}

// Patches of one half chunk for items with many entries (weights holding
// exact zeros, say): each lane stores its 8 decoded fragments at its slots
// (frag_index order) of `fb`, the lanes store the exact bf16 values of the
// half's entries [jlo, jhi) over their slots, 32 at a time, and each lane
// reads its fragments back.  Called by the whole warp.
__device__ __forceinline__ void patch_half_dense(StepFrag (&f)[8], uint4 *fb, const ItemPatches &ip, int jlo,
                                                 int jhi, int lane) {
    __syncwarp();   // earlier reads of fb's memory by any lane are done
#pragma unroll
    for (int J = 0; J < 8; ++J) fb[J * 32 + (lane ^ J)] = make_uint4(f[J].a0, f[J].a1, f[J].a2, f[J].a3);
    __syncwarp();
    uint16_t *fb16 = reinterpret_cast<uint16_t *>(fb);
    // all of the half's entries are requested before any is stored (one
    // round trip whether staged in shared memory or read from L2)
    for (int j0 = jlo; j0 < jhi; j0 += 8 * 32) {
        uint32_t ent[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int j = j0 + 32 * k + lane;
            ent[k] = j < jhi ? ip.entry(j) : 0u;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (j0 + 32 * k + lane < jhi) fb16[ent[k] & 0x7FFu] = (uint16_t)(ent[k] >> 16);
    }
    __syncwarp();
#pragma unroll
    for (int J = 0; J < 8; ++J) {
        const uint4 v = fb[J * 32 + (lane ^ J)];
        f[J] = StepFrag{v.x, v.y, v.z, v.w};
    }
}

template <int J>
__device__ __forceinline__ void decode_half(StepFrag (&f)[8], const uint32_t (&smA)[8], const uint32_t (&dA)[4],
                                            uint32_t eA, const uint32_t (&smB)[8], const uint32_t (&dB)[4],
                                            uint32_t eB) {
    f[J] = decode_step<J>(smA, dA, eA, smB, dB, eB);
    if constexpr (J + 1 < 8) decode_half<J + 1>(f, smA, dA, eA, smB, dB, eB);
}

// mma steps J..7 of one half chunk, batch <= 8: B = x[g][group + 4J .. +3],
// loaded 16 bytes at a time for steps J and J+1 by the lanes whose
// activation row g exists (the B operand of the others is zero).  Even and
// odd steps accumulate separately: two independent mma chains.
template <int J>
__device__ __forceinline__ void half_mma(const StepFrag (&f)[8], const uint16_t *xq, bool hasx, float (&ce)[4],
                                         float (&co)[4], uint4 bx = uint4{}) {
    if constexpr ((J & 1) == 0) bx = lds128_if(xq + 4 * J, hasx);
    float(&c)[4] = (J & 1) ? co : ce;
    if constexpr ((J & 1) == 0) mma_bf16_16816(c[0], c[1], c[2], c[3], f[J].a0, f[J].a1, f[J].a2, f[J].a3, bx.x, bx.y);
    else mma_bf16_16816(c[0], c[1], c[2], c[3], f[J].a0, f[J].a1, f[J].a2, f[J].a3, bx.z, bx.w);
    if constexpr (J + 1 < 8) half_mma<J + 1>(f, xq, hasx, ce, co, bx);
}

// The same for 9..16 rows of activations: each A fragment feeds two mma,
// one per group of 8 activation rows (x rows g and 8+g).
template <int J>
__device__ __forceinline__ void half_mma2(const StepFrag (&f)[8], const uint16_t *xq, const uint16_t *xq2,
                                          float (&ce)[4], float (&co)[4], float (&de)[4], float (&dd)[4]) {
    const uint2 b = *reinterpret_cast<const uint2 *>(xq + 4 * J);
    const uint2 b2 = *reinterpret_cast<const uint2 *>(xq2 + 4 * J);
    float(&c)[4] = (J & 1) ? co : ce;
    float(&d)[4] = (J & 1) ? dd : de;
    mma_bf16_16816(c[0], c[1], c[2], c[3], f[J].a0, f[J].a1, f[J].a2, f[J].a3, b.x, b.y);
    mma_bf16_16816(d[0], d[1], d[2], d[3], f[J].a0, f[J].a1, f[J].a2, f[J].a3, b2.x, b2.y);
    if constexpr (J + 1 < 8) half_mma2<J + 1>(f, xq, xq2, ce, co, de, dd);
}

// GGUF form: an item's activation rows (those below the batch) rewritten in
// place in the pair order of the decoded registers: word P of each
// 32-column group = (x[P], x[P + 16]).  Lane l handles words 4 (l % 4) .. +3
// of group l / 4; every lane loads before any stores.  Called by the warp.
template <int BMAX>
__device__ __forceinline__ void gguf_pair_order_x(uint16_t *xs, int batch, int lane) {
    const int q = lane >> 2, u = lane & 3;
    for (int b = 0; b < BMAX && b < batch; ++b) {
        uint16_t *grp = xs + b * kChunkElems + 32 * q;
        const uint2 lo = *reinterpret_cast<const uint2 *>(grp + 4 * u);
        const uint2 hi = *reinterpret_cast<const uint2 *>(grp + 16 + 4 * u);
        __syncwarp();
        *reinterpret_cast<uint4 *>(grp + 8 * u) = make_uint4(prmt(lo.x, hi.x, 0x5410u), prmt(lo.x, hi.x, 0x7632u),
                                                             prmt(lo.y, hi.y, 0x5410u), prmt(lo.y, hi.y, 0x7632u));
    }
    __syncwarp();
}

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

// One output value (b, row of this launch's rows): into y, or with the
// collective epilogue into every rank's exchange buffer as one 64-bit word
// whose high half is the launch epoch -- a single-copy-atomic store, so a
// reader that sees the epoch sees the value with it, and no fence is needed.
template <bool COLL>
__device__ __forceinline__ void store_y(const GemvParams &p, int b, int64_t row, float o, uint32_t epoch) {
    if constexpr (!COLL) {
        const int64_t idx = (int64_t)b * p.ldy + row;
        if (p.y_f32) reinterpret_cast<float *>(p.y)[idx] = o;
        else reinterpret_cast<uint16_t *>(p.y)[idx] = f32_to_bf16_bits_rn(o);
    } else {
        const int64_t w = p.mode == 0 ? (int64_t)b * p.ll_ld + p.row0 + row
                                      : ((int64_t)p.rank * p.batch + b) * p.ll_ld + row;
        const uint64_t v = (uint64_t)epoch << 32 | __float_as_uint(o);
        for (int q = 0; q < p.nranks; ++q) st_relaxed_sys_u64(p.ll[q] + w, v);
    }
}

// End of the collective epilogue, run by every warp of every CTA once it has
// sent its outputs, the warps that had no items too.  The [batch][out_total]
// outputs are dealt to all warps of the grid in equal contiguous ranges; a
// warp waits (bounded) for the words of its range in this GPU's exchange
// buffer to carry this launch's epoch and writes y from them.  Nothing here
// waits for anything but words that other warps send unconditionally, so no
// wait can close a cycle.  The warps then count themselves per CTA and the
// CTAs per GPU; the GPU's last CTA records the epoch for the next launch
// (read after griddepcontrol.wait, i.e. after this kernel has completed).
// A warp that gave up on a wait never counts itself, so the epoch does not
// advance and the following launches report timeouts until the caller resets
// the state.
template <int NW>
__device__ __forceinline__ void collective_finish(const GemvParams &p, uint32_t *cta_done, int warp, int lane,
                                                  uint32_t epoch) {
    const int64_t n_out = (int64_t)p.batch * p.out_total;
    const int64_t tw = (int64_t)gridDim.x * NW, wi = (int64_t)blockIdx.x * NW + warp;
    const int64_t o_lo = n_out * wi / tw, o_hi = n_out * (wi + 1) / tw;
    const uint64_t *mine = p.ll[p.rank];
    const int nsrc = p.mode == 0 ? 1 : p.nranks;
    bool ok = true;
    for (int64_t o = o_lo + lane; o < o_hi; o += 32) {
        const int b = (int)(o / p.out_total);
        const int64_t r = o - (int64_t)b * p.out_total;
        float acc = 0.f;
        for (int q = 0; q < nsrc; ++q) {
            const int64_t w = p.mode == 0 ? (int64_t)b * p.ll_ld + r : ((int64_t)q * p.batch + b) * p.ll_ld + r;
            uint32_t bits = 0;
            ok = ll_wait(mine + w, epoch, bits) && ok;
            acc += __uint_as_float(bits);
        }
        const int64_t idx = (int64_t)b * p.ldy + r;
        if (p.y_f32) reinterpret_cast<float *>(p.y)[idx] = acc;
        else reinterpret_cast<uint16_t *>(p.y)[idx] = f32_to_bf16_bits_rn(acc);
    }
    if (!__all_sync(0xffffffffu, ok)) return;
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) {
        __threadfence_block();
        old = atomicAdd(cta_done, 1u);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + 1 != (uint32_t)NW) return;
    if (lane == 0 && atomicAdd(p.state, 1u) + 1 == gridDim.x) {
        p.state[0] = 0u;
        p.state[1] = epoch;
    }
}

// Warp w of the partition owns items [T*w/W, T*(w+1)/W); item i belongs to
// warp floor(((i+1)*W - 1) / T).
__device__ __forceinline__ int64_t item_lo(int64_t w, int64_t T, int64_t W) { return T * w / W; }
__device__ __forceinline__ int64_t item_owner(int64_t i, int64_t T, int64_t W) { return ((i + 1) * W - 1) / T; }

template <int BMAX, int NW, bool XRES, bool COLL, int FMT = kFmtResident>
__global__ void __launch_bounds__(GemvCfg<BMAX, NW, XRES, FMT>::kWarps * 32, GemvCfg<BMAX, NW, XRES, FMT>::kCtasPerSm)
    gemv_kernel(const __grid_constant__ GemvParams p) {
    using C = GemvCfg<BMAX, NW, XRES, FMT>;
    constexpr bool GG = C::kGguf;
    constexpr int S = C::kStages;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // the weight slots want a 1024-byte-aligned base (128-byte swizzle)
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff) + warp * S;
    int64_t *rec_of = reinterpret_cast<int64_t *>(smem + C::kRecOff) + warp * S;
    uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + C::kBarOff) + C::kWarps * S;
    for (int i = threadIdx.x; i < 128; i += blockDim.x) reinterpret_cast<uint32_t *>(smem + C::kZeroOff)[i] = 0u;
    if (threadIdx.x == 0) *reinterpret_cast<uint32_t *>(smem + C::kCtaOff) = 0u;
    if (lane == 0)
        for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    if (XRES && threadIdx.x == 0) mbar_init(xbar, 1);
    fence_mbar_init();
    __syncthreads();
    griddep_launch_dependents();

    const int64_t gw = (int64_t)blockIdx.x * C::kWarps + warp;
    uint32_t *cta_done = reinterpret_cast<uint32_t *>(smem + C::kCtaOff);           // warps of the CTA finished
    if (gw >= p.W) {
        if constexpr (COLL) {
            griddep_wait();
            collective_finish<C::kWarps>(p, cta_done, warp, lane, *reinterpret_cast<volatile uint32_t *>(p.state + 1) + 1u);
        }
        return;
    }
    if (lane == 0) {
        prefetch_tensormap(&p.wmap);
        prefetch_tensormap(&p.xmap);
    }
    const int64_t lo = item_lo(gw, p.T, p.W), hi = item_lo(gw + 1, p.T, p.W);
    const int64_t first_tile = lo / p.nch;
    uint8_t *wsm = smem + C::kWOff + warp * S * C::kWBytes;      // this warp's weight slots
    uint8_t *xrs = smem + C::kXROff + warp * S * C::kXRSlot;     // its activation + record slots
    const uint16_t *zero_x = reinterpret_cast<const uint16_t *>(smem + C::kZeroOff);

    // ---- issue the copies of item (tile, c) into slot `s`: lane 0 alone,
    // three TMA operations (16 weight rows, the activation slice, the record)
    auto issue = [&](int64_t tile, int c, int s, int32_t r_off, int32_t r_end) {
        if (lane == 0) {
            const int staged = GG && !p.has_rec ? 0 : min(r_end - r_off, C::kPcap);
            uint8_t *xr = xrs + s * C::kXRSlot;
            rec_of[s] = r_off;
            mbar_arrive_expect_tx(&bars[s], (uint32_t)(C::kWBytes + (XRES ? 0 : BMAX * kXRowBytes) + staged * 4));
            if constexpr (GG) tma_load_2d(wsm + s * C::kWBytes, &p.wmap, c * kGgufChunkWords, (int)(tile * kTileRows), &bars[s]);
            else tma_load_4d(wsm + s * C::kWBytes, &p.wmap, 0, 0, c, (int)(tile * kTileRows), &bars[s]);
            if constexpr (!XRES) tma_load_2d(xr, &p.xmap, c * kChunkElems, 0, &bars[s]);
            if (staged > 0) bulk_g2s(xr + C::kPOff, p.precs + r_off, (uint32_t)staged * 4, &bars[s]);
        }
    };

    // issue cursor: the next item to be copied, as (tile, chunk) and index;
    // its record bounds are loaded one refill ahead of their use
    int64_t i_it = lo, i_tile = first_tile;
    int i_c = (int)(lo - first_tile * p.nch);
    int32_t nxt_off = 0, nxt_end = 0;
    uint32_t epoch = 0;                           // collective epilogue only
    const bool has_rec = !GG || p.has_rec;
    auto load_rec = [&]() {
        if (i_it < hi && has_rec) {
            nxt_off = __ldg(p.ptile_off + i_it);
            nxt_end = __ldg(p.ptile_off + i_it + 1);
        }
    };
    auto advance_issue = [&]() {
        ++i_it;
        if (++i_c == p.nch) { i_c = 0; ++i_tile; }
    };
    {
        // First S items.  Everything read from the weight (rows, records,
        // record offsets) is requested before griddep_wait, so it overlaps
        // the end of the previous kernel of the stream; the activations, the
        // outputs and the scratch are touched only after it.  Each slot's
        // expected bytes are raised without arriving; the activation copy's
        // arrival completes the phase.  The weight rows go first: they need
        // no record offset, so their copies are in flight while the offsets
        // load.
        int64_t tl = i_tile;
        int cc = i_c;
        for (int s = 0; s < S && lo + s < hi; ++s) {
            if (lane == 0) {
                mbar_expect_tx(&bars[s], (uint32_t)C::kWBytes);
                if constexpr (GG) tma_load_2d(wsm + s * C::kWBytes, &p.wmap, cc * kGgufChunkWords, (int)(tl * kTileRows), &bars[s]);
                else tma_load_4d(wsm + s * C::kWBytes, &p.wmap, 0, 0, cc, (int)(tl * kTileRows), &bars[s]);
            }
            if (++cc == p.nch) { cc = 0; ++tl; }
        }
        const int32_t v = (has_rec && lane <= S + 1 && lo + lane <= p.T) ? __ldg(p.ptile_off + lo + lane) : 0;
        for (int s = 0; s < S && lo + s < hi; ++s) {
            const int32_t r_off = __shfl_sync(0xffffffffu, v, s), r_end = __shfl_sync(0xffffffffu, v, s + 1);
            if (lane == 0) {
                const int staged = min(r_end - r_off, C::kPcap);
                rec_of[s] = r_off;
                if constexpr (XRES) mbar_arrive_expect_tx(&bars[s], (uint32_t)(staged * 4));
                else if (staged > 0) mbar_expect_tx(&bars[s], (uint32_t)(staged * 4));
                if (staged > 0) bulk_g2s(xrs + s * C::kXRSlot + C::kPOff, p.precs + r_off, (uint32_t)staged * 4, &bars[s]);
            }
        }
        griddep_wait();
        // this launch's epoch (the previous launch on this GPU recorded its own)
        if constexpr (COLL) epoch = *reinterpret_cast<volatile uint32_t *>(p.state + 1) + 1u;
        if constexpr (XRES) {
            if (warp == 0 && lane == 0) {
                mbar_arrive_expect_tx(xbar, (uint32_t)(p.nch * BMAX * kXRowBytes));
                for (int c2 = 0; c2 < p.nch; ++c2)
                    tma_load_2d(smem + C::kXCOff + c2 * BMAX * kXRowBytes, &p.xmap, c2 * kChunkElems, 0, xbar);
            }
            for (int s = 0; s < S && i_it < hi; ++s) advance_issue();
            if (!mbar_wait(xbar, 0u, &g_status)) return;
        } else {
            for (int s = 0; s < S && i_it < hi; ++s) {
                if (lane == 0) {
                    mbar_arrive_expect_tx(&bars[s], (uint32_t)(BMAX * kXRowBytes));
                    tma_load_2d(xrs + s * C::kXRSlot, &p.xmap, i_c * kChunkElems, 0, &bars[s]);
                }
                advance_issue();
            }
        }
        nxt_off = __shfl_sync(0xffffffffu, v, S);
        nxt_end = __shfl_sync(0xffffffffu, v, S + 1);
    }

    const int g = lane >> 2, t = lane & 3;
    // shared-memory offsets of this lane's groups t (half 0) and 4 + t
    // (half 1) of row g in a staged item; row g + 8 is 8 x 384 bytes further
    const GroupOffsets go[2] = {sw_group_offsets((uint32_t)g, (uint32_t)t), sw_group_offsets((uint32_t)g, 4u + t)};
    constexpr int kRowB = 8 * kChunkBytes;
    constexpr int BW = BMAX > 8 ? 16 : 8;           // activation rows per partial-sum row
    constexpr int PW = 16 * BW;                     // floats per partial
    float ce[4] = {0.f, 0.f, 0.f, 0.f}, co[4] = {0.f, 0.f, 0.f, 0.f};
    float de[4] = {0.f, 0.f, 0.f, 0.f}, dd[4] = {0.f, 0.f, 0.f, 0.f};   // rows 8..15 (BMAX > 8)
    float pc[4] = {0.f, 0.f, 0.f, 0.f}, pd[4] = {0.f, 0.f, 0.f, 0.f};   // patch corrections
    int64_t tile = first_tile;
    int c = (int)(lo - first_tile * p.nch);
    int tile_c0 = c;                                // first chunk of the current tile in this range
    int s = 0;
    uint32_t parity = 0;

    // Split tiles: every piece's warp publishes its partial sums and counts
    // itself on the tile's counter; the warp that brings the count to the
    // number of pieces sums them in warp order (deterministic) and writes y.
    auto pieces_before = [&](int64_t tl) -> int {
        return (int)(item_owner(tl * p.nch + p.nch - 1, p.T, p.W) - item_owner(tl * p.nch, p.T, p.W));
    };
    auto reduce_split = [&](int64_t tl) {
        const int64_t w_first = item_owner(tl * p.nch, p.T, p.W);
        const int64_t w_last = item_owner(tl * p.nch + p.nch - 1, p.T, p.W);
        // w_first's piece is in its slot 1 when its range began in an earlier
        // tile; every later warp's range begins in this tile: slot 0
        const int sl_first = item_lo(w_first, p.T, p.W) < tl * p.nch ? 1 : 0;
        constexpr int KN = PW / 32;                 // values per lane
        constexpr int KB = KN > 4 ? 4 : 8;          // pieces loaded per round
        const int np = (int)(w_last - w_first) + 1;
        float o4[KN];
#pragma unroll
        for (int k = 0; k < KN; ++k) o4[k] = 0.f;
        // all pieces of a round are requested before any is added (one L2
        // round trip per round), then summed in warp order (deterministic)
        for (int b0 = 0; b0 < np; b0 += KB) {
            float v[KB][KN];
#pragma unroll
            for (int u = 0; u < KB; ++u) {
                const int i = b0 + u;
                const float *src = p.partials + ((w_first + i) * 2 + (i == 0 ? sl_first : 0)) * PW + lane;
#pragma unroll
                for (int k = 0; k < KN; ++k) v[u][k] = i < np ? __ldcg(src + 32 * k) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < KB; ++u)
#pragma unroll
                for (int k = 0; k < KN; ++k) o4[k] += v[u][k];
        }
        const int64_t row0 = tl * kTileRows;
#pragma unroll
        for (int k = 0; k < KN; ++k) {
            const int idx = lane + 32 * k;
            const int rr = idx / BW, b = idx % BW;
            float o = o4[k];
            const int64_t row = row0 + rr;
            if (b < p.batch && row < p.rows) {
                if (p.bias) o += bf16_bits_to_f32(__ldg(p.bias + row));
                store_y<COLL>(p, b, row, o, epoch);
            }
        }
        if (lane == 0) p.tile_cnt[tl] = 0;
    };

    for (int64_t it = lo; it < hi; ++it) {
        if (!mbar_wait(&bars[s], parity, &g_status)) return;
        const uint8_t *wsl = wsm + s * C::kWBytes;
        const uint8_t *xr = xrs + s * C::kXRSlot;
        const uint16_t *xs = reinterpret_cast<const uint16_t *>(XRES ? smem + C::kXCOff + c * BMAX * kXRowBytes : xr);
        if constexpr (!GG) {
            const uint32_t *rec = reinterpret_cast<const uint32_t *>(xr + C::kPOff);
            const uint32_t hdr = rec[kRecHdr];
            const uint2 ewA = *reinterpret_cast<const uint2 *>(rec + 2 * g);        // emax of row g, groups 0..7
            const uint2 ewB = *reinterpret_cast<const uint2 *>(rec + 2 * g + 16);   // row g + 8
            const uint16_t *xg = g < BMAX ? xs + g * kChunkElems : zero_x;
            // both halves' compressed groups are read up front, so the
            // shared-memory latency overlaps the first half's decode
            uint32_t smA[2][8], dA[2][4], smB[2][8], dB[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                load_group_sw(wsl, go[h], smA[h], dA[h]);
                load_group_sw(wsl + kRowB, go[h], smB[h], dB[h]);
            }
            const ItemPatches ip{rec, p.precs, rec_of + s, C::kPcap, C::kRecHdrW};
            const int n_low = (int)(hdr & 0xFFFFu), n_all = (int)(hdr >> 16);
            // Few entries (the usual case): the patched weights enter the
            // products with their saturated value, and (exact - saturated) * x
            // is added to the correction sums of their rows, in entry order
            // (deterministic), while the compressed groups are still on their
            // way from shared memory.  Many entries: the fragments go through
            // shared memory, where the exact values are stored over them.
            const bool dense = n_all > kSparseEntries;
            if (!dense) {
                // entry `lane`, decoded by its lane: row << 8 | column, delta
                uint32_t pkey = 0u;
                float pdv = 0.f;
                if (lane < n_all) {
                    const uint32_t ent = ip.entry(lane);
                    uint32_t rr, cc;
                    frag_position(ent, rr, cc);
                    pkey = rr << 8 | cc;
                    pdv = patch_delta(ent, rec_emax(rec, (int)rr, (int)(cc >> 5)));
                }
                for (int e = 0; e < n_all; e += 2) {      // two entries per pass: independent chains
                    const uint32_t k0 = __shfl_sync(0xffffffffu, pkey, e), k1 = __shfl_sync(0xffffffffu, pkey, e + 1);
                    const float v0 = __shfl_sync(0xffffffffu, pdv, e), v1 = __shfl_sync(0xffffffffu, pdv, e + 1);
                    add_patch<BMAX>(k0, v0, true, g, t, xs, pc, pd);
                    add_patch<BMAX>(k1, v1, e + 1 < n_all, g, t, xs, pc, pd);
                }
            }
            // the two halves: decode, patch (dense items), multiply; the
            // dense path is a separate copy so the usual one stays straight
            auto halves = [&](auto dense_tag) {
                constexpr bool kDense = decltype(dense_tag)::value;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t eA = emax_x2(((h ? ewA.y : ewA.x) >> (8 * t)) & 0xFFu);
                    const uint32_t eB = emax_x2(((h ? ewB.y : ewB.x) >> (8 * t)) & 0xFFu);
                    StepFrag f[8];
                    decode_half<0>(f, smA[h], dA[h], eA, smB[h], dB[h], eB);
                    // the item's compressed rows are in registers by now, so
                    // their slot serves as the 4 KB fragment buffer
                    if constexpr (kDense)
                        patch_half_dense(f, reinterpret_cast<uint4 *>(const_cast<uint8_t *>(wsl)), ip, h ? n_low : 0,
                                         h ? n_all : n_low, lane);
                    const int q = 4 * h + t;
                    if constexpr (BMAX > 8) {
                        half_mma2<0>(f, xg + 32 * q, xs + (8 + g) * kChunkElems + 32 * q, ce, co, de, dd);
                    } else {
                        half_mma<0>(f, xg + 32 * q, g < BMAX, ce, co);
                    }
                }
            };
            if (dense) halves(std::true_type{});
            else halves(std::false_type{});
            // shared-memory writes of the generic proxy before the slot's
            // refill by the TMA engine (async proxy)
            if (dense) fence_proxy_async_smem();
        } else {
            // GGUF blocks: the activations into the decoded pair order, the
            // four 12-word windows of the lane's blocks (rows g and g + 8,
            // blocks 2t and 2t + 1 of the chunk) into registers, then per
            // half: decode, side-table values (dense), multiply.
            gguf_pair_order_x<BMAX>(reinterpret_cast<uint16_t *>(const_cast<uint8_t *>(xr)), p.batch, lane);
            const uint32_t *rec = reinterpret_cast<const uint32_t *>(xr + C::kPOff);
            const uint32_t hdr = p.has_rec ? rec[0] : 0u;
            const uint16_t *xg = g < BMAX ? xs + g * kChunkElems : zero_x;
            const uint32_t *wv = reinterpret_cast<const uint32_t *>(wsl);
            uint32_t wA[2][12], wB[2][12];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int i = 0; i < 12; ++i) {
                    wA[h][i] = wv[g * kGgufChunkWords + 23 * t + 11 * h + i];
                    wB[h][i] = wv[(g + 8) * kGgufChunkWords + 23 * t + 11 * h + i];
                }
            // blocks with an emax below 7 (never written by the packer, and
            // the zero rows past the end of the weight) take the exact
            // per-lane form, for the whole warp
            const uint32_t emin = min(min(gguf_min_emax<0>(wA[0]), gguf_min_emax<0>(wB[0])),
                                      min(gguf_min_emax<1>(wA[1]), gguf_min_emax<1>(wB[1])));
            const bool exact_form = __any_sync(0xffffffffu, emin < 7u);
            const ItemPatches ip{rec, p.precs, rec_of + s, C::kPcap, C::kRecHdrW};
            const int n_low = (int)(hdr & 0xFFFFu), n_all = (int)(hdr >> 16);
            auto half = [&](auto h_tag, auto fast_tag) {
                constexpr int h = decltype(h_tag)::value;
                constexpr bool kFast = decltype(fast_tag)::value;
                uint32_t pa[16], pb[16];
                gguf_pairs_from<0, kFast>(gguf_load_block<h>(wA[h]), pa);
                gguf_pairs_from<0, kFast>(gguf_load_block<h>(wB[h]), pb);
                StepFrag f[8];
#pragma unroll
                for (int J = 0; J < 8; ++J) f[J] = StepFrag{pa[2 * J], pb[2 * J], pa[2 * J + 1], pb[2 * J + 1]};
                // the windows are in registers, so the weight slot serves as
                // the fragment buffer of the side-table values
                if (n_all > 0)
                    patch_half_dense(f, reinterpret_cast<uint4 *>(const_cast<uint8_t *>(wsl)), ip, h ? n_low : 0,
                                     h ? n_all : n_low, lane);
                const int q = 2 * t + h;
                if constexpr (BMAX > 8) {
                    half_mma2<0>(f, xg + 32 * q, xs + (8 + g) * kChunkElems + 32 * q, ce, co, de, dd);
                } else {
                    half_mma<0>(f, xg + 32 * q, g < BMAX, ce, co);
                }
            };
            using I0 = std::integral_constant<int, 0>;
            using I1 = std::integral_constant<int, 1>;
            if (exact_form) {
                half(I0{}, std::false_type{});
                half(I1{}, std::false_type{});
            } else {
                half(I0{}, std::true_type{});
                half(I1{}, std::true_type{});
            }
            // the permuted activations and side-table values were written
            // with generic stores before the slot's refill by the TMA engine
            fence_proxy_async_smem();
        }

        // ---- refill this slot S items ahead
        __syncwarp();
        // the slot was only read with ordinary loads, which have completed
        // (their values are consumed), so the bulk copies may overwrite it
        if (i_it < hi) {
            issue(i_tile, i_c, s, nxt_off, nxt_end);
            advance_issue();
            load_rec();
        }

        // ---- tile finished (or range ends inside it)
        if (c == p.nch - 1 || it == hi - 1) {
            const float c0 = ce[0] + co[0] + pc[0], c1 = ce[1] + co[1] + pc[1];
            const float c2 = ce[2] + co[2] + pc[2], c3 = ce[3] + co[3] + pc[3];
            const float d0 = de[0] + dd[0] + pd[0], d1 = de[1] + dd[1] + pd[1];
            const float d2 = de[2] + dd[2] + pd[2], d3 = de[3] + dd[3] + pd[3];
            const int64_t row0 = tile * kTileRows;
            const bool whole = tile_c0 == 0 && c == p.nch - 1;
            if (whole) {
                const float v[8] = {c0, c1, c2, c3, d0, d1, d2, d3};
#pragma unroll
                for (int k = 0; k < (BMAX > 8 ? 8 : 4); ++k) {
                    const int64_t row = row0 + g + 8 * ((k >> 1) & 1);
                    const int b = 2 * t + (k & 1) + 8 * (k >> 2);
                    if (b < p.batch && row < p.rows) {
                        float o = v[k];
                        if (p.bias) o += bf16_bits_to_f32(__ldg(p.bias + row));
                        store_y<COLL>(p, b, row, o, epoch);
                    }
                }
            } else {
                // partial tile: publish this piece, the last arriving warp reduces
                const int pslot = tile == first_tile ? 0 : 1;
                float *mine = p.partials + (gw * 2 + pslot) * PW;
                *reinterpret_cast<float2 *>(mine + g * BW + 2 * t) = make_float2(c0, c1);
                *reinterpret_cast<float2 *>(mine + (g + 8) * BW + 2 * t) = make_float2(c2, c3);
                if constexpr (BMAX > 8) {
                    *reinterpret_cast<float2 *>(mine + g * BW + 8 + 2 * t) = make_float2(d0, d1);
                    *reinterpret_cast<float2 *>(mine + (g + 8) * BW + 8 + 2 * t) = make_float2(d2, d3);
                }
                // the warp's stores, then one acquire-release count: it publishes
                // them to whichever warp arrives last and, for that warp,
                // orders its reads of the other pieces after the count
                __syncwarp();
                int old = 0;
                if (lane == 0)
                    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.tile_cnt + tile) : "memory");
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == pieces_before(tile)) {
                    __syncwarp();
                    reduce_split(tile);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) ce[k] = co[k] = de[k] = dd[k] = pc[k] = pd[k] = 0.f;
            tile_c0 = 0;
        }
        if (++s == S) { s = 0; parity ^= 1u; }
        if (++c == p.nch) { c = 0; ++tile; }
    }
    if constexpr (COLL) collective_finish<C::kWarps>(p, cta_done, warp, lane, epoch);
}

struct GemvLaunch {
    int grid;
    int64_t W, T;
    int n_tiles, nch;
};

static int device_sms() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = sms > 0 ? sms : 1;
    }
    return cache[dev];
}

// Small cache of encoded tensor maps: encoding is host work that would be
// repeated on every call for the same weight and activation buffers.
struct MapKey {
    const void *ptr;
    int64_t a, b, c;
    int dev;
    bool operator==(const MapKey &o) const { return ptr == o.ptr && a == o.a && b == o.b && c == o.c && dev == o.dev; }
};

static bool cached_map(CUtensorMap *out, const MapKey &key, bool (*make)(CUtensorMap *, const MapKey &)) {
    constexpr int kSlots = 256;
    static MapKey keys[kSlots];
    static CUtensorMap maps[kSlots];
    static bool used[kSlots] = {false};
    static std::mutex mu;
    const size_t h = (reinterpret_cast<uintptr_t>(key.ptr) >> 8) ^ (size_t)(key.a * 31 + key.b * 7 + key.c + key.dev);
    const int slot = (int)(h % kSlots);
    std::lock_guard<std::mutex> lk(mu);
    if (used[slot] && keys[slot] == key) {
        *out = maps[slot];
        return true;
    }
    if (!make(out, key)) return false;
    keys[slot] = key;
    maps[slot] = *out;
    used[slot] = true;
    return true;
}

static bool make_wmap(CUtensorMap *m, const MapKey &k) {   // a = rows, b = in_f
    const int64_t nch = (k.b + kChunkElems - 1) / kChunkElems;
    return encode_resident_map(m, k.ptr, k.a, nch, resident_row_bytes(k.b), kTileRows);
}

static bool make_xmap(CUtensorMap *m, const MapKey &k) {   // a = in_pad, b = batch, c = ldx | bmax << 40
    const int64_t ldx = k.c & ((1ll << 40) - 1), bmax = k.c >> 40;
    const cuuint64_t dims[2] = {(cuuint64_t)k.a, (cuuint64_t)k.b};
    const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kChunkElems, (cuuint32_t)bmax};
    return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, k.ptr, dims, strides, box);
}

static GemvLaunch plan_gemv(int64_t rows, int64_t in_f, int nw) {
    GemvLaunch L;
    L.nch = (int)((in_f + kChunkElems - 1) / kChunkElems);
    L.n_tiles = (int)((rows + kTileRows - 1) / kTileRows);
    L.T = (int64_t)L.n_tiles * L.nch;
    const int64_t want = (L.T + nw - 1) / nw;
    const int ctas_per_sm = nw == 6 ? 2 : 1;       // GemvCfg<...,6>::kCtasPerSm
    L.grid = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)device_sms() * ctas_per_sm, want));
    L.W = std::min<int64_t>((int64_t)L.grid * nw, L.T);
    return L;
}

// Warps per CTA for a launch: 12 (more items in flight per SM) unless that
// splits a tile (16 rows x all chunks) into more than about 8 warps' pieces,
// whose split-tile reduction then costs more than the extra warps gain.
// Batch 1 below 32768 items (the decoder's q/k/v, o, down projections): the
// same 12 warps per SM as two CTAs of 6, each with half the shared memory, so
// that when a CTA finishes, a CTA of the next GEMV of the stream fits beside
// its sibling and starts fetching its weights (programmatic dependent launch)
// while this launch's last pieces finish: the chain of small launches in a
// decode step overlaps (1B decoder 1.607 -> 1.570 ms per token; the 4-shape
// bench step unchanged).  The collective epilogue keeps one CTA of 12, and
// above 8 rows its activation slots.
// 5..8 rows: 12 with the CTA's activation block (in_f <= 4096 and enough
// items to repay its copy), else 10, else 8; above 8 rows 12 with the CTA's
// activation block under the same condition (one slot per warp), else 8
// (7 fit).
static bool xres_for(int64_t T, int64_t nch) { return nch <= kXResChunks && T >= 8192; }

static int warps_for(int64_t batch, int64_t rows, int64_t in_f, bool coll = false) {
    const int64_t nch = (in_f + kChunkElems - 1) / kChunkElems;
    const int64_t T = (rows + kTileRows - 1) / kTileRows * nch;
    const bool wide = T * 8 >= nch * (int64_t)device_sms() * 12;
    if (batch == 1) return wide ? (T < 32768 && !coll ? GemvCfg<1, 6>::kWarps : GemvCfg<1, 12>::kWarps) : GemvCfg<1, 8>::kWarps;
    if (batch == 2) return wide ? GemvCfg<2, 12>::kWarps : GemvCfg<2, 8>::kWarps;
    if (batch <= 4) return wide ? GemvCfg<4, 12>::kWarps : GemvCfg<4, 8>::kWarps;
    if (batch <= 8)
        return wide ? (xres_for(T, nch) ? GemvCfg<8, 12, true>::kWarps : GemvCfg<8, 10>::kWarps) : GemvCfg<8, 8>::kWarps;
    return xres_for(T, nch) && !coll ? GemvCfg<16, 12, true>::kWarps : GemvCfg<16, 8>::kWarps;
}

// The GGUF form: the same choice without the CTA activation block.
static int warps_for_gguf(int64_t batch, int64_t rows, int64_t in_f) {
    const int64_t nch = (in_f + kChunkElems - 1) / kChunkElems;
    const int64_t T = (rows + kTileRows - 1) / kTileRows * nch;
    const bool wide = T * 8 >= nch * (int64_t)device_sms() * 12;
    if (batch == 1) return wide ? GemvCfg<1, 16, false, kFmtGguf>::kWarps : GemvCfg<1, 8, false, kFmtGguf>::kWarps;
    if (batch == 2) return wide ? GemvCfg<2, 12, false, kFmtGguf>::kWarps : GemvCfg<2, 8, false, kFmtGguf>::kWarps;
    if (batch <= 4) return wide ? GemvCfg<4, 12, false, kFmtGguf>::kWarps : GemvCfg<4, 8, false, kFmtGguf>::kWarps;
    if (batch <= 8) return wide ? GemvCfg<8, 10, false, kFmtGguf>::kWarps : GemvCfg<8, 8, false, kFmtGguf>::kWarps;
    return GemvCfg<16, 8, false, kFmtGguf>::kWarps;
}

// partial sums: per unit two [16][8] (batch <= 8) or [16][16] fp32 slots
static int64_t scratch_need(const GemvLaunch &L, int64_t batch) { return L.W * 2 * 16 * (batch > 8 ? 16 : 8) * 4; }

template <int BMAX, int NW, bool XRES, bool COLL, int FMT = kFmtResident>
static int launch_gemv_as(const GemvParams &p, const GemvLaunch &L, cudaStream_t st) {
    using C = GemvCfg<BMAX, NW, XRES, FMT>;
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64] = {false};
    if (dev < 0 || dev >= 64) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv: device index %d", dev);
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<BMAX, NW, XRES, COLL, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemv: smem attribute: %s", cudaGetErrorString(e));
        attr_set[dev] = true;
    }
    // programmatic stream serialization: this launch may begin while the
    // previous kernel of the stream finishes (see griddep_wait in the kernel)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)L.grid);
    cfg.blockDim = dim3((unsigned)(C::kWarps * 32));
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_kernel<BMAX, NW, XRES, COLL, FMT>, p);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemv: launch: %s", cudaGetErrorString(e));
    return check_launch("bf16x_gemv");
}

// The plain GEMV and the collective-epilogue one are separate instantiations,
// so the plain kernel carries no trace of the peer stores.
template <int BMAX, int NW, bool XRES = false>
static int launch_gemv(const GemvParams &p, const GemvLaunch &L, cudaStream_t st) {
    return p.nranks > 1 ? launch_gemv_as<BMAX, NW, XRES, true>(p, L, st) : launch_gemv_as<BMAX, NW, XRES, false>(p, L, st);
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int64_t bf16x_gemv_scratch_bytes(int64_t rows, int64_t in_f) {
    if (rows <= 0 || in_f <= 0) return 0;
    int64_t need = 0;
    for (int b : {1, 2, 4, 8, 16}) need = std::max(need, scratch_need(plan_gemv(rows, in_f, warps_for(b, rows, in_f)), b));
    return need;
}

namespace bf16x {

// Destinations of the collective epilogue (bf16x_gemv_peers); none for the
// plain GEMV.
struct PeerArgs {
    int nranks, rank, mode;
    uint64_t *const *ll;
    int64_t ll_ld, out_total, row0;
    uint32_t *state;
};

static int gemv_impl(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                     int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                     const uint16_t *bias, void *y, int y_dtype, int64_t ldy,
                     int32_t *tile_counters, void *scratch, int64_t scratch_bytes, void *stream,
                     const PeerArgs *peers);

}  // namespace bf16x

extern "C" int bf16x_gemv(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                          int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                          const uint16_t *bias, void *y, int y_dtype, int64_t ldy,
                          int32_t *tile_counters, void *scratch, int64_t scratch_bytes, void *stream) {
    return gemv_impl(layout, ptile_off, precs, rows, in_f, x, batch, ldx, bias, y, y_dtype, ldy, tile_counters,
                     scratch, scratch_bytes, stream, nullptr);
}

extern "C" int bf16x_gemv_peers(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                                int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                                const uint16_t *bias, int mode, uint64_t *const *ll, int64_t ll_ld,
                                int64_t out_total, int64_t row0, int nranks, int rank, void *y, int y_dtype,
                                int64_t ldy, uint32_t *state, int32_t *tile_counters, void *scratch,
                                int64_t scratch_bytes, void *stream) {
    if (nranks < 2 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: need 2 <= nranks <= %d and 0 <= rank < nranks", kMaxRanks);
    if (mode != 0 && mode != 1) return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: mode must be 0 (gather) or 1 (reduce)");
    if (!ll || !state || !y) return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: null exchange table, state or y");
    for (int q = 0; q < nranks; ++q) {
        if (!ll[q]) return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: null exchange buffer for rank %d", q);
        if (reinterpret_cast<uintptr_t>(ll[q]) & 7u)
            return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: exchange buffers must be 8-byte aligned");
    }
    if (rows <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: every rank needs rows (its peers wait for its words)");
    if (mode == 0 && (row0 < 0 || row0 + rows > out_total))
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: rows [row0, row0+rows) outside 0..out_total");
    if (mode == 1 && (rows != out_total || row0 != 0))
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: reduce mode takes every output row (rows == out_total, row0 == 0)");
    if (ll_ld < out_total || ldy < out_total)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv_peers: ll_ld and ldy must be >= out_total");
    const PeerArgs pa{nranks, rank, mode, ll, ll_ld, out_total, row0, state};
    return gemv_impl(layout, ptile_off, precs, rows, in_f, x, batch, ldx, bias, y, y_dtype, ldy,
                     tile_counters, scratch, scratch_bytes, stream, &pa);
}

namespace bf16x {

static int gemv_impl(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                     int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                     const uint16_t *bias, void *y, int y_dtype, int64_t ldy,
                     int32_t *tile_counters, void *scratch, int64_t scratch_bytes, void *stream,
                     const PeerArgs *peers) {
    if (rows < 0 || in_f <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: bad shape");
    if (in_f > 65536) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv: in_f > 65536");
    if (batch < 1 || batch > 16) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: batch must be 1..16 (got %lld)", (long long)batch);
    if (y_dtype != BF16X_DTYPE_BF16 && y_dtype != BF16X_DTYPE_F32)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: bad y_dtype");
    if (rows == 0) return BF16X_OK;
    if (!layout || !ptile_off || !precs || !x || !y) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: null pointer");
    const int64_t in_pad = (in_f + kChunkElems - 1) / kChunkElems * kChunkElems;
    if (ldx < in_pad || (ldx % 8) != 0)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: ldx must be a multiple of 8 and >= %lld (zero padded)", (long long)in_pad);
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(layout) | reinterpret_cast<uintptr_t>(precs)) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: x, layout and records must be 16-byte aligned");
    if (ldy < rows && !peers) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: ldy < rows");
    const int nw = warps_for(batch, rows, in_f, peers != nullptr);
    const GemvLaunch L = plan_gemv(rows, in_f, nw);
    if (!tile_counters) return set_error(BF16X_ERR_INVALID, "bf16x_gemv: tile_counters (ceil(rows/16) zeroed int32) missing");
    if (!scratch || scratch_bytes < scratch_need(L, batch))
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: scratch of %lld bytes needed", (long long)scratch_need(L, batch));
    if (reinterpret_cast<uintptr_t>(scratch) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv: scratch must be 16-byte aligned");
    GemvParams p = {};
    {
        int dev = 0;
        cudaGetDevice(&dev);
        const int64_t bmax = batch == 1 ? 1 : batch == 2 ? 2 : batch <= 4 ? 4 : batch <= 8 ? 8 : 16;
        if (!cached_map(&p.wmap, MapKey{layout, rows, in_f, 0, dev}, make_wmap))
            return set_error(BF16X_ERR_CUDA, "bf16x_gemv: weight tensor map");
        if (!cached_map(&p.xmap, MapKey{x, in_pad, batch, ldx | (bmax << 40), dev}, make_xmap))
            return set_error(BF16X_ERR_CUDA, "bf16x_gemv: activation tensor map");
    }
    p.layout = layout; p.ptile_off = ptile_off; p.precs = precs;
    p.rows = rows; p.row_bytes = resident_row_bytes(in_f);
    p.has_rec = 1;
    p.nch = L.nch; p.n_tiles = L.n_tiles; p.T = L.T; p.W = L.W;
    p.x = x; p.ldx = ldx; p.batch = (int)batch;
    p.bias = bias; p.y = y; p.y_f32 = y_dtype == BF16X_DTYPE_F32; p.ldy = ldy;
    p.tile_cnt = tile_counters;
    p.partials = static_cast<float *>(scratch);
    p.nranks = 1;
    p.rank = 0;
    p.state = nullptr;
    if (peers) {
        p.nranks = peers->nranks;
        p.rank = peers->rank;
        p.mode = peers->mode;
        for (int q = 0; q < peers->nranks; ++q) p.ll[q] = peers->ll[q];
        p.ll_ld = peers->ll_ld;
        p.out_total = peers->out_total;
        p.row0 = peers->row0;
        p.state = peers->state;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (batch == 1) return nw == 6 ? launch_gemv<1, 6>(p, L, st) : nw > 8 ? launch_gemv<1, 12>(p, L, st) : launch_gemv<1, 8>(p, L, st);
    if (batch == 2) return nw > 8 ? launch_gemv<2, 12>(p, L, st) : launch_gemv<2, 8>(p, L, st);
    if (batch <= 4) return nw > 8 ? launch_gemv<4, 12>(p, L, st) : launch_gemv<4, 8>(p, L, st);
    if (batch <= 8) {
        if (nw <= 8) return launch_gemv<8, 8>(p, L, st);
        return xres_for(L.T, L.nch) ? launch_gemv<8, 12, true>(p, L, st) : launch_gemv<8, 10>(p, L, st);
    }
    return xres_for(L.T, L.nch) && p.nranks == 1 ? launch_gemv<16, 12, true>(p, L, st) : launch_gemv<16, 8>(p, L, st);
}

}  // namespace bf16x

// ------------------------------------------------------- GGUF-block GEMV
namespace bf16x {

static bool make_gguf_map(CUtensorMap *m, const MapKey &k) {   // a = rows, b = in_f
    const int64_t rb = gguf_row_bytes(k.b);
    const cuuint64_t dims[2] = {(cuuint64_t)(rb / 4), (cuuint64_t)k.a};
    const cuuint64_t strides[1] = {(cuuint64_t)rb};
    const cuuint32_t box[2] = {(cuuint32_t)kGgufChunkWords, (cuuint32_t)kTileRows};
    return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, k.ptr, dims, strides, box);
}

}  // namespace bf16x

extern "C" int64_t bf16x_gguf_gemv_scratch_bytes(int64_t rows, int64_t in_f) {
    if (rows <= 0 || in_f <= 0) return 0;
    int64_t need = 0;
    for (int b : {1, 2, 4, 8, 16})
        need = std::max(need, scratch_need(plan_gemv(rows, in_f, warps_for_gguf(b, rows, in_f)), b));
    return need;
}

extern "C" int bf16x_gguf_gemv(const uint8_t *blocks, int64_t rows, int64_t in_f, const int32_t *item_off,
                               const uint32_t *item_recs, const uint16_t *x, int64_t batch, int64_t ldx,
                               const uint16_t *bias, void *y, int y_dtype, int64_t ldy, int32_t *tile_counters,
                               void *scratch, int64_t scratch_bytes, void *stream) {
    if (rows < 0 || in_f <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: bad shape");
    if (in_f % kChunkElems != 0 || in_f > 65536)
        return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gguf_gemv: in_f must be a multiple of 256 and <= 65536 (got %lld)",
                         (long long)in_f);
    if (batch < 1 || batch > 16) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: batch must be 1..16 (got %lld)", (long long)batch);
    if (y_dtype != BF16X_DTYPE_BF16 && y_dtype != BF16X_DTYPE_F32)
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: bad y_dtype");
    if ((item_off == nullptr) != (item_recs == nullptr))
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: side-table offsets and records go together");
    if (rows == 0) return BF16X_OK;
    if (!blocks || !x || !y) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: null pointer");
    if (ldx < in_f || (ldx % 8) != 0)
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: ldx must be a multiple of 8 and >= in_f");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(blocks) | reinterpret_cast<uintptr_t>(item_recs)) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: x, blocks and records must be 16-byte aligned");
    if (ldy < rows) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: ldy < rows");
    const int nw = warps_for_gguf(batch, rows, in_f);
    const GemvLaunch L = plan_gemv(rows, in_f, nw);
    if (!tile_counters) return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: tile_counters (ceil(rows/16) zeroed int32) missing");
    if (!scratch || scratch_bytes < scratch_need(L, batch))
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: scratch of %lld bytes needed", (long long)scratch_need(L, batch));
    if (reinterpret_cast<uintptr_t>(scratch) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_gguf_gemv: scratch must be 16-byte aligned");
    GemvParams p = {};
    {
        int dev = 0;
        cudaGetDevice(&dev);
        const int64_t bmax = batch == 1 ? 1 : batch == 2 ? 2 : batch <= 4 ? 4 : batch <= 8 ? 8 : 16;
        if (!cached_map(&p.wmap, MapKey{blocks, rows, in_f, 1, dev}, make_gguf_map))
            return set_error(BF16X_ERR_CUDA, "bf16x_gguf_gemv: block tensor map");
        if (!cached_map(&p.xmap, MapKey{x, in_f, batch, ldx | (bmax << 40), dev}, make_xmap))
            return set_error(BF16X_ERR_CUDA, "bf16x_gguf_gemv: activation tensor map");
    }
    p.layout = blocks; p.ptile_off = item_off; p.precs = item_recs;
    p.has_rec = item_off != nullptr;
    p.rows = rows; p.row_bytes = gguf_row_bytes(in_f);
    p.nch = L.nch; p.n_tiles = L.n_tiles; p.T = L.T; p.W = L.W;
    p.x = x; p.ldx = ldx; p.batch = (int)batch;
    p.bias = bias; p.y = y; p.y_f32 = y_dtype == BF16X_DTYPE_F32; p.ldy = ldy;
    p.tile_cnt = tile_counters;
    p.partials = static_cast<float *>(scratch);
    p.nranks = 1;
    cudaStream_t st = (cudaStream_t)stream;
    constexpr int G = kFmtGguf;
    if (batch == 1) return nw > 8 ? launch_gemv_as<1, 16, false, false, G>(p, L, st) : launch_gemv_as<1, 8, false, false, G>(p, L, st);
    if (batch == 2) return nw > 8 ? launch_gemv_as<2, 12, false, false, G>(p, L, st) : launch_gemv_as<2, 8, false, false, G>(p, L, st);
    if (batch <= 4) return nw > 8 ? launch_gemv_as<4, 12, false, false, G>(p, L, st) : launch_gemv_as<4, 8, false, false, G>(p, L, st);
    if (batch <= 8) return nw > 8 ? launch_gemv_as<8, 10, false, false, G>(p, L, st) : launch_gemv_as<8, 8, false, false, G>(p, L, st);
    return launch_gemv_as<16, 8, false, false, G>(p, L, st);
}

// ------------------------------------------------ no-allocation GEMV entry
// bf16x_gemv_noalloc serves callers that cannot hand this library device
// memory: a plain C host or FFI binding with no device allocator of its own,
// or a serving loop that must not call cudaMalloc/cudaFree (they synchronise
// the device) once it is running.  Its tile counters and partial sums live in
// one fixed, file-scope device array instead of caller-owned buffers.
namespace bf16x {

constexpr int64_t kNoAllocMaxTiles = 32768;                   // rows <= 524288
constexpr int64_t kNoAllocCounterBytes = kNoAllocMaxTiles * 4;  // 128 KiB
constexpr int64_t kNoAllocPartialBytes = 2ll << 20;           // 2 MiB: 2048 warps x 1 KiB
constexpr int64_t kNoAllocBytes = kNoAllocCounterBytes + kNoAllocPartialBytes;

static __device__ __align__(256) unsigned char g_gemv_noalloc_scratch[kNoAllocBytes];

// Device address of g_gemv_noalloc_scratch on the current device, looked up
// once per device (with that device current) and cached.
static int noalloc_scratch(void **out) {
    static void *addr[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemv_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv_noalloc: device index %d", dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(BF16X_ERR_CUDA, "bf16x_gemv_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return BF16X_OK;
}

}  // namespace bf16x

extern "C" int64_t bf16x_gemv_noalloc_max_rows(void) { return kNoAllocMaxTiles * kTileRows; }

extern "C" int bf16x_gemv_noalloc(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                                  int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                                  const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *stream) {
    if (rows < 0 || in_f <= 0) return set_error(BF16X_ERR_INVALID, "bf16x_gemv_noalloc: bad shape");
    if (in_f > 65536) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv_noalloc: in_f > 65536");
    if (batch < 1 || batch > 8)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemv_noalloc: batch must be 1..8 (got %lld)", (long long)batch);
    if (rows == 0) return BF16X_OK;
    const int64_t n_tiles = (rows + kTileRows - 1) / kTileRows;
    if (n_tiles > kNoAllocMaxTiles)
        return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemv_noalloc: rows %lld exceed the fixed scratch limit of %lld",
                         (long long)rows, (long long)(kNoAllocMaxTiles * kTileRows));
    const int64_t need = scratch_need(plan_gemv(rows, in_f, warps_for(batch, rows, in_f)), batch);
    if (need > kNoAllocPartialBytes)
        return set_error(BF16X_ERR_UNSUPPORTED,
                         "bf16x_gemv_noalloc: %lld bytes of partial sums needed, fixed scratch holds %lld",
                         (long long)need, (long long)kNoAllocPartialBytes);
    void *base = nullptr;
    if (int rc = noalloc_scratch(&base)) return rc;
    // The counters must be zero at launch; a call that failed part-way could
    // have left some set, so clear this call's range every time.
    int32_t *counters = static_cast<int32_t *>(base);
    cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)n_tiles * 4, (cudaStream_t)stream);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemv_noalloc: clearing counters: %s", cudaGetErrorString(e));
    return bf16x_gemv(layout, ptile_off, precs, rows, in_f, x, batch, ldx, bias, y, y_dtype, ldy, counters,
                      static_cast<unsigned char *>(base) + kNoAllocCounterBytes, kNoAllocPartialBytes, stream);
}
