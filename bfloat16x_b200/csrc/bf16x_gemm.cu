// bf16x_gemm.cu -- fused BF16X decode + GEMM on the 5th-generation tensor
// cores (tcgen05 / TMEM), sm_100a.
//
// Replaces _bf16x_gemm_fused_kernel / bf16x_fused_gemm
// (bf16x_gemm_fused.py:31-114), and unlike it applies the exact-delta
// patches, so the product equals the matmul with the exact bf16 weights.
//
//   y[m][n] = sum_k x[m][k] * W[n][k] (+ bias[n])
//
// One persistent CTA per SM walks output tiles of 128 weight rows x BN tokens.
// The MMA is D[128 rows][BN tokens] += A[128][64] * B[BN][64]^T per k-block of
// 64 columns: A = the decoded weights, B = the activations, both K-major
// 128-byte-swizzled in shared memory, D in tensor memory.
//
// Warp roles (23 warps):
//   0      W producer: per 256-column chunk, TMAs of kGemmWRows rows x 384
//          bytes of the resident layout (128 rows by default: one stage per
//          chunk, in a ring of stages; 128-byte swizzled) + the 16-row patch
//          records of the stage (the groups' emax and the patch entries)
//   1      B producer: one swizzled TMA per k-block (BN rows x 64 columns)
//   2      MMA issuer: TMEM allocation, 4 x tcgen05.mma (K=16) per k-block,
//          tcgen05.commit to release the A and B slots and to publish a tile
//   3..18  decoders, two groups of 8 alternating k-blocks: each k-block
//          (128 x 64 weights) is decoded from the compressed chunk into the
//          swizzled A slot (five integer ops per pair), patched with the
//          exact values, fenced for the async proxy
//   19..22 epilogue: tcgen05.ld of the fp32 accumulator (each warp its TMEM
//          lane quarter = 32 weight rows), bias, coalesced transposed stores
// The accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of one tile overlaps the MMAs of the next.  Every wait is bounded;
// a role that gives up raises the shared abort flag, every role then leaves
// its loop, and TMEM is released before the kernel returns.
#include <algorithm>
#include <mutex>

#include <cuda_runtime.h>

#include "bf16x_common.cuh"
#include "bf16x_resident.cuh"
#include "bf16x_status.cuh"
#include "bf16x_tmap.h"
#include "bf16x_wait.cuh"

namespace bf16x {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmDecWarps = 16;                  // two groups of 8, alternating k-blocks
constexpr int kGemmThreads = (3 + kGemmDecWarps + 4) * 32;
constexpr int kGemmRecCap = 192;                     // record words staged per 16-row sub-tile
#ifndef BF16X_GEMM_WROWS
#define BF16X_GEMM_WROWS 128
#endif
constexpr int kGemmWRows = BF16X_GEMM_WROWS;          // weight rows per compressed stage
constexpr int kWHalves = kGemmBM / kGemmWRows;        // compressed stages per chunk
constexpr int kSubsPerStage = kGemmWRows / 16;        // 16-row patch records per stage
constexpr int kGemmWStage = kGemmWRows * kChunkBytes;

template <int BN>
struct GemmCfg {
    static constexpr int kWStages = kWHalves == 2 ? 3 : 2;   // ring of compressed stages
    static constexpr int kAStages = 3;
    static constexpr int kBStages = BN >= 256 ? (kWHalves == 2 ? 3 : 2) : 4;
    static constexpr int kAStage = kGemmBM * 128;     // 16 KB
    static constexpr int kBStage = BN * 128;
    static constexpr int kRecStage = kSubsPerStage * kGemmRecCap * 4;   // the 16-row records of a stage
    static constexpr int kAOff = 0;                                       // 1024-aligned slots first
    static constexpr int kBOff = kAOff + kAStages * kAStage;
    static constexpr int kWOff = kBOff + kBStages * kBStage;
    static constexpr int kROff = kWOff + kWStages * kGemmWStage;
    static constexpr int kBarOff = kROff + kWStages * kRecStage;
    // barriers: w_full, w_empty, a_full, a_empty, b_full, b_empty, acc_full, acc_empty (2)
    static constexpr int kNumBars = 2 * kWStages + 2 * kAStages + 2 * kBStages + 4;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;               // tmem base, abort flag
    static constexpr int kSmem = kMiscOff + 16 + 1024;                    // + alignment slack
    static constexpr int kTmemCols = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct GemmParams {
    CUtensorMap wmap;    // resident layout [rows][chunks][3 lines], box kGemmWRows rows x 1 chunk, 128B swizzle
    CUtensorMap xmap;    // activations [M][in_f] bf16, box BN rows x 64 columns, 128B swizzle
    const int32_t *ptile_off;
    const uint32_t *precs;
    int64_t rows, M;
    int nch, n_tiles16;
    int tiles_n, tiles_total;
    const uint16_t *bias;
    void *y;
    int y_f32;
    int64_t ldy;
};

// ------------------------------------------------------------- tcgen05 glue
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    // K-major, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);          // start address
    d |= (uint64_t)1u << 16;                               // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;                     // stride byte offset
    d |= (uint64_t)1u << 46;                               // descriptor version (sm100)
    d |= (uint64_t)2u << 61;                               // layout: SWIZZLE_128B
    return d;
}

template <int BN>
__host__ __device__ constexpr uint32_t umma_idesc_bf16() {
    return (1u << 4)                       // D: f32
         | (1u << 7)                       // A: bf16
         | (1u << 10)                      // B: bf16
         | ((uint32_t)(BN >> 3) << 17)     // N
         | ((uint32_t)(kGemmBM >> 4) << 24);   // M = 128
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory");
}

// Byte offset of element (row, col) inside a 128-row x 64-column K-major
// 128-byte-swizzled tile (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col) {
    return row * 128u + ((((col >> 3) ^ row) & 7u) << 4) + ((col & 7u) << 1);
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ GemmParams p) {
    using C = GemmCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand slots
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
    uint64_t *w_full = bars, *w_empty = w_full + C::kWStages;
    uint64_t *a_full = w_empty + C::kWStages, *a_empty = a_full + C::kAStages;
    uint64_t *b_full = a_empty + C::kAStages, *b_empty = b_full + C::kBStages;
    uint64_t *acc_full = b_empty + C::kBStages, *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kWStages; ++s) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], kGemmDecWarps / kWHalves); }
        for (int s = 0; s < C::kAStages; ++s) { mbar_init(&a_full[s], 8); mbar_init(&a_empty[s], 1); }
        for (int s = 0; s < C::kBStages; ++s) { mbar_init(&b_full[s], 1); mbar_init(&b_empty[s], 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 4); }
        abort_flag[0] = 0;
        abort_flag[1] = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(C::kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int nkb = p.nch * 4;                     // k-blocks per tile

    if (warp == 0) {
        // ------------------------------------------------------- W producer
        // Stages are (tile, chunk, half) in order; the record offsets of the
        // next stage are loaded while the current one is issued, so their
        // global-memory latency stays off the critical path.
        if (lane == 0) {
            prefetch_tensormap(&p.wmap);
            int ws = 0;
            uint32_t wph = 0;
            const int per_tile = p.nch * kWHalves;
            int t = blockIdx.x, c = 0, hf = 0;
            int32_t off[kSubsPerStage], len[kSubsPerStage];
            auto load_offsets = [&](int tt, int cc, int hh) {
                const int rt = tt / p.tiles_n;
#pragma unroll
                for (int sub = 0; sub < kSubsPerStage; ++sub) {
                    const int64_t t16 = (int64_t)rt * 8 + kSubsPerStage * hh + sub;
                    if (tt < p.tiles_total && t16 < p.n_tiles16) {
                        const int64_t i = t16 * p.nch + cc;
                        off[sub] = __ldg(p.ptile_off + i);
                        len[sub] = __ldg(p.ptile_off + i + 1);
                    } else {
                        off[sub] = 0;
                        len[sub] = 0;
                    }
                }
            };
            load_offsets(t, c, hf);
            (void)per_tile;
            while (t < p.tiles_total) {
                int32_t o[kSubsPerStage], l[kSubsPerStage];
                int total = 0;
#pragma unroll
                for (int sub = 0; sub < kSubsPerStage; ++sub) {
                    o[sub] = off[sub];
                    l[sub] = min(len[sub] - off[sub], kGemmRecCap);
                    total += l[sub];
                }
                const int rt = t / p.tiles_n, cc = c, hh = hf;
                // advance to the next stage and prefetch its offsets
                if (++hf == kWHalves) { hf = 0; if (++c == p.nch) { c = 0; t += gridDim.x; } }
                load_offsets(t, c, hf);
                if (!role_wait(&w_empty[ws], wph ^ 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&w_full[ws], (uint32_t)(kGemmWStage + total * 4));
                tma_load_4d(smem + C::kWOff + ws * kGemmWStage, &p.wmap, 0, 0, cc, rt * kGemmBM + kGemmWRows * hh,
                            &w_full[ws]);
                uint8_t *rec = smem + C::kROff + ws * C::kRecStage;
#pragma unroll
                for (int sub = 0; sub < kSubsPerStage; ++sub)
                    if (l[sub] > 0)
                        bulk_g2s(rec + sub * kGemmRecCap * 4, p.precs + o[sub], (uint32_t)l[sub] * 4, &w_full[ws]);
                if (++ws == C::kWStages) { ws = 0; wph ^= 1u; }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- B producer
        if (lane == 0) {
            prefetch_tensormap(&p.xmap);
            int bs = 0;
            uint32_t bph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.tiles_total && ok; t += gridDim.x) {
                const int nt = t % p.tiles_n;
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!role_wait(&b_empty[bs], bph ^ 1u, abort_flag)) { ok = false; break; }
                    mbar_arrive_expect_tx(&b_full[bs], (uint32_t)C::kBStage);
                    tma_load_2d(smem + C::kBOff + bs * C::kBStage, &p.xmap, kb * kGemmBK, nt * BN, &b_full[bs]);
                    if (++bs == C::kBStages) { bs = 0; bph ^= 1u; }
                }
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16<BN>();
            int as = 0, bs = 0, ac = 0;
            uint32_t aph = 0, bph = 0, acph = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.tiles_total && ok; t += gridDim.x) {
                if (!role_wait(&acc_empty[ac], acph ^ 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ac * BN);
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!role_wait(&a_full[as], aph, abort_flag) || !role_wait(&b_full[bs], bph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = umma_desc_sw128(smem_u32(smem + C::kAOff + as * C::kAStage));
                    const uint64_t bd = umma_desc_sw128(smem_u32(smem + C::kBOff + bs * C::kBStage));
#pragma unroll
                    for (int k16 = 0; k16 < kGemmBK / 16; ++k16)   // 32 bytes along K per step
                        umma_bf16(d_tmem, ad + 2u * k16, bd + 2u * k16, idesc, (kb | k16) != 0);
                    umma_commit(&a_empty[as]);
                    umma_commit(&b_empty[bs]);
                    if (++as == C::kAStages) { as = 0; aph ^= 1u; }
                    if (++bs == C::kBStages) { bs = 0; bph ^= 1u; }
                }
                if (!ok) break;
                umma_commit(&acc_full[ac]);
                if (++ac == 2) { ac = 0; acph ^= 1u; }
            }
        }
    } else if (warp < 3 + kGemmDecWarps) {
        // ------------------------------------------------------- decoders
        // Two groups of 8 warps take alternate k-blocks, so two k-blocks are
        // decoded at once.  Warp d of a group owns weight rows 16d..16d+15:
        // two lanes per row (32 columns each of the 64-column k-block), and
        // the patch record of that 16-row sub-tile, whose entries for the
        // k-block are one contiguous range (records are sorted by 64-column
        // quarter).  Everything a warp writes it also patches, so warps
        // never wait for each other; each arrives on the MMA barrier on its
        // own (count 8 per k-block, 16 per chunk for the W slot).
        const int dg = (warp - 3) >> 3, d = (warp - 3) & 7;
        const int hf = d / kSubsPerStage;              // which stage of the chunk holds my rows
        const int lrow = 16 * (d % kSubsPerStage) + (lane >> 1);   // row inside that stage
        const int row = 16 * d + (lane >> 1), hh = lane & 1;
        int as = 0, wseq = 0;
        uint32_t aph = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < p.tiles_total && ok; t += gridDim.x) {
            const int rt = t / p.tiles_n;
            const bool has_rec = (int64_t)rt * 8 + d < p.n_tiles16;
            for (int c = 0; c < p.nch && ok; ++c, wseq += kWHalves) {
                const int wslot = (wseq + hf) % C::kWStages;
                const uint32_t wpar = (uint32_t)(((wseq + hf) / C::kWStages) & 1);
                const uint8_t *wst = smem + C::kWOff + wslot * kGemmWStage;
                const uint32_t *rec = reinterpret_cast<const uint32_t *>(smem + C::kROff + wslot * C::kRecStage) +
                                      (d % kSubsPerStage) * kGemmRecCap;
                // this warp's patch entries for its two quarters of the chunk
                // (k-blocks dg and dg+2): lane j holds entries j and 32+j of
                // each, read from the staged record once the chunk has landed
                int qlo[2] = {0, 0}, qn[2] = {0, 0};
                uint32_t qe[2][2] = {{0u, 0u}, {0u, 0u}};
                for (int kq = 0; kq < 4; ++kq) {
                    const bool mine = (kq & 1) == dg;
                    if (mine) {
                        int w = 1;
                        if (lane == 0) {
                            if (kq == dg) w = role_wait(&w_full[wslot], wpar, abort_flag);
                            w = w && role_wait(&a_empty[as], aph ^ 1u, abort_flag);
                        }
                        w = __shfl_sync(0xffffffffu, w, 0);
                        if (!w) { ok = false; break; }
                        if (kq == dg && has_rec) {
                            // quarter boundaries 0 | n_q0 | n_low | n_q012 | n_all
                            const uint32_t h0 = rec[kRecHdr], h1 = rec[kRecHdr + 1];
                            const int bq[5] = {0, (int)(h1 & 0xFFFFu), (int)(h0 & 0xFFFFu), (int)(h1 >> 16), (int)(h0 >> 16)};
#pragma unroll
                            for (int u = 0; u < 2; ++u) {
                                const int q = dg + 2 * u;
                                const int lo = q == 0 ? bq[0] : q == 1 ? bq[1] : q == 2 ? bq[2] : bq[3];
                                const int hi = q == 0 ? bq[1] : q == 1 ? bq[2] : q == 2 ? bq[3] : bq[4];
                                qlo[u] = lo;
                                qn[u] = hi - lo;
                                const int j0 = kRecHdrWords + lo + lane;
                                qe[u][0] = (lane < qn[u] && j0 < kGemmRecCap) ? rec[j0] : 0u;
                                qe[u][1] = (lane + 32 < qn[u] && j0 + 32 < kGemmRecCap) ? rec[j0 + 32] : 0u;
                            }
                        }
                        uint8_t *ast = smem + C::kAOff + as * C::kAStage;
                        {
                            // row `row`, columns 64*kq + 32*hh .. +31 of the chunk
                            uint32_t sm[8], dw[4];
                            load_group_sw(wst, sw_group_offsets((uint32_t)lrow, (uint32_t)(2 * kq + hh)), sm, dw);
                            const uint32_t e2 = has_rec ? emax_x2(rec_emax(rec, lane >> 1, 2 * kq + hh)) : 0u;
                            GroupPairs gp;
                            decode_pairs_from<0>(gp, sm, dw, e2);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t col = 32u * hh + 8u * i;
                                *reinterpret_cast<uint4 *>(ast + sw128_offset((uint32_t)row, col)) =
                                    make_uint4(gp.w[4 * i], gp.w[4 * i + 1], gp.w[4 * i + 2], gp.w[4 * i + 3]);
                            }
                        }
                        __syncwarp();
                        if (has_rec) {
                            // exact values of this sub-tile's patched weights in the k-block
                            const int u = kq == dg ? 0 : 1;
                            const int n = u ? qn[1] : qn[0], lo = u ? qlo[1] : qlo[0];
                            auto put = [&](uint32_t ent) {
                                uint32_t rr, cc;
                                frag_position(ent, rr, cc);
                                *reinterpret_cast<uint16_t *>(ast + sw128_offset(16u * d + rr, cc & 63u)) =
                                    (uint16_t)(ent >> 16);
                            };
                            const int cap = kGemmRecCap - kRecHdrWords - lo;   // entries staged in shared memory
                            if (lane < n && lane < cap) put(u ? qe[1][0] : qe[0][0]);
                            if (lane + 32 < n && lane + 32 < cap) put(u ? qe[1][1] : qe[0][1]);
                            if (n > 64 || cap < n) {
                                // past the staged words or past 64 entries: from global memory
                                const int32_t base = __ldg(p.ptile_off + ((int64_t)rt * 8 + d) * p.nch + c);
                                for (int j = lane; j < n; j += 32)
                                    if (j >= 64 || j >= cap) put(__ldg(p.precs + base + kRecHdrWords + lo + j));
                            }
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[as]);
                    }
                    if (++as == C::kAStages) { as = 0; aph ^= 1u; }
                }
                if (!ok) break;
                if (lane == 0) mbar_arrive(&w_empty[wslot]);
            }
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int qd = warp & 3;                       // TMEM lane quarter
        int ac = 0;
        uint32_t acph = 0;
        for (int t = blockIdx.x; t < p.tiles_total; t += gridDim.x) {
            if (!role_wait(&acc_full[ac], acph, abort_flag)) break;
            tc_fence_after();
            const int rt = t / p.tiles_n, nt = t % p.tiles_n;
            const int64_t row = (int64_t)rt * kGemmBM + 32 * qd + lane;
            const float bias = (p.bias && row < p.rows) ? bf16_bits_to_f32(__ldg(p.bias + row)) : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem_base + ((uint32_t)(32 * qd) << 16) + (uint32_t)(ac * BN + c0), v);
                if (row < p.rows) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int64_t n = (int64_t)nt * BN + c0 + i;
                        if (n < p.M) {
                            const float o = __uint_as_float(v[i]) + bias;
                            if (p.y_f32) reinterpret_cast<float *>(p.y)[n * p.ldy + row] = o;
                            else reinterpret_cast<uint16_t *>(p.y)[n * p.ldy + row] = f32_to_bf16_bits_rn(o);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ac]);
            if (++ac == 2) { ac = 0; acph ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem_base), "r"(C::kTmemCols) : "memory");
    }
}


// ------------------------------------------------ CTA-pair (cluster of 2) glue
// BN = tokens per pair tile: 256 (each CTA stages 128; two accumulators, so
// the epilogue of one tile overlaps the next) or 512 (each CTA stages 256;
// two N=256 MMAs per decoded k-block fill the whole of tensor memory, one
// accumulator) -- the latter decodes every weight once per 512 tokens.
template <int BN>
struct Gemm2Cfg {
    static constexpr int kWStages = 2;
    static constexpr int kAStages = BN > 256 ? 3 : 4;
    static constexpr int kBStages = BN > 256 ? 2 : 3;
    static constexpr int kAccBufs = BN > 256 ? 1 : 2;
    static constexpr int kAStage = kGemmBM * 128;     // 16 KB: 128 rows x 64 columns
    static constexpr int kBStage = (BN / 2) * 128;    // this CTA's BN/2 tokens x 64 columns
    static constexpr int kRecStage = kSubsPerStage * kGemmRecCap * 4;
    static constexpr int kAOff = 0;
    static constexpr int kBOff = kAOff + kAStages * kAStage;
    static constexpr int kWOff = kBOff + kBStages * kBStage;
    static constexpr int kROff = kWOff + kWStages * kGemmWStage;
    static constexpr int kBarOff = kROff + kWStages * kRecStage;
    static constexpr int kNumBars = 2 * kWStages + 3 * kAStages + 2 * kBStages + 4;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kSmem = kMiscOff + 16 + 1024;
    static constexpr int kTmemCols = 512;             // two 256-column accumulators, or one of 512
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

// Relaxed arrival on a barrier of another CTA of the cluster: the ordering
// that matters is already established by the caller (see its use).
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;"
                 :: "r"(cluster_addr), "r"(bytes) : "memory");
}

// Tiled TMA load into this CTA's shared memory whose completion is counted
// on a barrier of the leader CTA of the pair (a plain load of this CTA's half).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const void *map, int c0, int c1, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(bar_cluster) : "memory");
}

template <int M, int N>
__host__ __device__ constexpr uint32_t umma_idesc_bf16_m() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// Arrive on the barrier at this shared-memory offset in BOTH CTAs of the
// pair (ctaMask 0b11) once the pair's MMAs issued so far have completed: one
// commit instead of one per CTA.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(smem_u32(bar)), "h"((uint16_t)3u) : "memory");
}

// All threads of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The CTA pair version (cluster of 2, tcgen05 cta_group::2): a tile is 256
// weight rows x 256 tokens; CTA r of the pair decodes rows 128r..128r+127
// and stages tokens 128r..128r+127 of the activations, and the leader
// (rank 0) issues M=256 x N=256 MMAs that read both CTAs' operands and write
// each CTA's 128 accumulator rows into its own tensor memory.  Per SM the
// activation traffic and its shared-memory ring are half those of the
// single-CTA kernel, which leaves room for a deeper ring of decoded tiles.
// All "full" barriers that the MMA waits on live in the leader; the MMA's
// commits release the slots of both CTAs; the epilogues of both CTAs
// release the leader's accumulator.
template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm2sm_kernel(const __grid_constant__ GemmParams p) {
    using C = Gemm2Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand slots
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
    uint64_t *w_full = bars, *w_empty = w_full + C::kWStages;
    uint64_t *a_full = w_empty + C::kWStages, *a_empty = a_full + C::kAStages;
    uint64_t *b_full = a_empty + C::kAStages, *b_empty = b_full + C::kBStages;
    uint64_t *acc_full = b_empty + C::kBStages, *acc_empty = acc_full + 2;
    uint64_t *a_ready = acc_empty + 2;             // peer only: its decoders' local count per A slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kWStages; ++s) { mbar_init(&w_full[s], 1); mbar_init(&w_empty[s], kGemmDecWarps / kWHalves); }
        // a_full: the leader's 8 decoder warps + one forwarded arrival for the peer's 8
        for (int s = 0; s < C::kAStages; ++s) { mbar_init(&a_full[s], 9); mbar_init(&a_empty[s], 1); mbar_init(&a_ready[s], 8); }
        // b_full: the leader's arrival carries the bytes of both halves
        for (int s = 0; s < C::kBStages; ++s) { mbar_init(&b_full[s], 1); mbar_init(&b_empty[s], 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 8); }
        abort_flag[0] = 0;
        abort_flag[1] = 0;
        fence_mbar_init();
    }
    // barriers of both CTAs initialised before any crosses the pair
    cluster_sync_all();
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(C::kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the leader's barrier addresses, as seen from this CTA
    auto leader = [&](uint64_t *bar) { return mapa_shared(smem_u32(bar), 0u); };
    const uint32_t tmem_base = *tmem_slot;
    const int nkb = p.nch * 4;                     // k-blocks per tile

    if (warp == 0) {
        // ------------------------------------------------------- W producer
        // Stages are (tile, chunk, half) in order; the record offsets of the
        // next stage are loaded while the current one is issued, so their
        // global-memory latency stays off the critical path.
        if (lane == 0) {
            prefetch_tensormap(&p.wmap);
            int ws = 0;
            uint32_t wph = 0;
            const int per_tile = p.nch * kWHalves;
            int t = pair, c = 0, hf = 0;
            int32_t off[kSubsPerStage], len[kSubsPerStage];
            auto load_offsets = [&](int tt, int cc, int hh) {
                const int rt = tt / p.tiles_n;
#pragma unroll
                for (int sub = 0; sub < kSubsPerStage; ++sub) {
                    const int64_t t16 = (int64_t)rt * 16 + 8 * rank + kSubsPerStage * hh + sub;
                    if (tt < p.tiles_total && t16 < p.n_tiles16) {
                        const int64_t i = t16 * p.nch + cc;
                        off[sub] = __ldg(p.ptile_off + i);
                        len[sub] = __ldg(p.ptile_off + i + 1);
                    } else {
                        off[sub] = 0;
                        len[sub] = 0;
                    }
                }
            };
            load_offsets(t, c, hf);
            (void)per_tile;
            while (t < p.tiles_total) {
                int32_t o[kSubsPerStage], l[kSubsPerStage];
                int total = 0;
#pragma unroll
                for (int sub = 0; sub < kSubsPerStage; ++sub) {
                    o[sub] = off[sub];
                    l[sub] = min(len[sub] - off[sub], kGemmRecCap);
                    total += l[sub];
                }
                const int rt = t / p.tiles_n, cc = c, hh = hf;
                // advance to the next stage and prefetch its offsets
                if (++hf == kWHalves) { hf = 0; if (++c == p.nch) { c = 0; t += npairs; } }
                load_offsets(t, c, hf);
                if (!role_wait(&w_empty[ws], wph ^ 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&w_full[ws], (uint32_t)(kGemmWStage + total * 4));
                tma_load_4d(smem + C::kWOff + ws * kGemmWStage, &p.wmap, 0, 0, cc,
                            rt * 2 * kGemmBM + (int)rank * kGemmBM + kGemmWRows * hh, &w_full[ws]);
                uint8_t *rec = smem + C::kROff + ws * C::kRecStage;
#pragma unroll
                for (int sub = 0; sub < kSubsPerStage; ++sub)
                    if (l[sub] > 0)
                        bulk_g2s(rec + sub * kGemmRecCap * 4, p.precs + o[sub], (uint32_t)l[sub] * 4, &w_full[ws]);
                if (++ws == C::kWStages) { ws = 0; wph ^= 1u; }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- B producer
        if (lane == 0) {
            prefetch_tensormap(&p.xmap);
            int bs = 0;
            uint32_t bph = 0;
            bool ok = true;
            for (int t = pair; t < p.tiles_total && ok; t += npairs) {
                const int nt = t % p.tiles_n;
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!role_wait(&b_empty[bs], bph ^ 1u, abort_flag)) { ok = false; break; }
                    // this CTA's half of the token tile, counted on the leader's barrier
                    const uint32_t lb = leader(&b_full[bs]);
                    if (rank == 0) mbar_arrive_expect_tx(&b_full[bs], (uint32_t)(2 * C::kBStage));
                    if constexpr (BN > 256) {
                        // tokens [r*128, +128) and [256 + r*128, +128) of the tile: the
                        // first and second N=256 MMA each read 128 tokens per CTA
                        tma_load_2d_pair(smem + C::kBOff + bs * C::kBStage, &p.xmap, kb * kGemmBK,
                                         nt * BN + (int)rank * 128, lb);
                        tma_load_2d_pair(smem + C::kBOff + bs * C::kBStage + 128 * 128, &p.xmap, kb * kGemmBK,
                                         nt * BN + 256 + (int)rank * 128, lb);
                    } else {
                        tma_load_2d_pair(smem + C::kBOff + bs * C::kBStage, &p.xmap, kb * kGemmBK,
                                         nt * BN + (int)rank * (BN / 2), lb);
                    }
                    if (++bs == C::kBStages) { bs = 0; bph ^= 1u; }
                }
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16_m<2 * kGemmBM, (BN > 256 ? 256 : BN)>();
            int as = 0, bs = 0, ac = 0;
            uint32_t aph = 0, bph = 0, acph = 0;
            bool ok = true;
            for (int t = pair; t < p.tiles_total && ok; t += npairs) {
                if (!role_wait(&acc_empty[ac], acph ^ 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ac * BN);
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!role_wait(&a_full[as], aph, abort_flag) || !role_wait(&b_full[bs], bph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = umma_desc_sw128(smem_u32(smem + C::kAOff + as * C::kAStage));
                    const uint64_t bd = umma_desc_sw128(smem_u32(smem + C::kBOff + bs * C::kBStage));
#pragma unroll
                    for (int k16 = 0; k16 < kGemmBK / 16; ++k16) {   // 32 bytes along K per step
                        umma_bf16_pair(d_tmem, ad + 2u * k16, bd + 2u * k16, idesc, (kb | k16) != 0);
                        if constexpr (BN > 256)   // tokens 256..511: the stage's rows 128..255 (16 KB on)
                            umma_bf16_pair(d_tmem + 256u, ad + 2u * k16, bd + (uint64_t)((128 * 128) >> 4) + 2u * k16,
                                           idesc, (kb | k16) != 0);
                    }
                    umma_commit_pair_both(&a_empty[as]);
                    umma_commit_pair_both(&b_empty[bs]);
                    if (++as == C::kAStages) { as = 0; aph ^= 1u; }
                    if (++bs == C::kBStages) { bs = 0; bph ^= 1u; }
                }
                if (!ok) break;
                umma_commit_pair_both(&acc_full[ac]);
                if (++ac == C::kAccBufs) { ac = 0; acph ^= 1u; }
            }
        }
        if (lane == 0 && rank == 1) {
            // peer: forward each k-block's "A slot decoded" count to the leader
            int as = 0;
            uint32_t aph = 0;
            bool ok = true;
            for (int t = pair; t < p.tiles_total && ok; t += npairs) {
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!role_wait(&a_ready[as], aph, abort_flag)) { ok = false; break; }
                    // the decoder warps fenced their tile for the async proxy before
                    // their local arrival, which this thread has acquired
                    mbar_arrive_cluster_relaxed(leader(&a_full[as]));
                    if (++as == C::kAStages) { as = 0; aph ^= 1u; }
                }
            }
        }
    } else if (warp < 3 + kGemmDecWarps) {
        // ------------------------------------------------------- decoders
        // Two groups of 8 warps take alternate k-blocks, so two k-blocks are
        // decoded at once.  Warp d of a group owns weight rows 16d..16d+15:
        // two lanes per row (32 columns each of the 64-column k-block), and
        // the patch record of that 16-row sub-tile, whose entries for the
        // k-block are one contiguous range (records are sorted by 64-column
        // quarter).  Everything a warp writes it also patches, so warps
        // never wait for each other; each arrives on the MMA barrier on its
        // own (count 8 per k-block, 16 per chunk for the W slot).
        const int dg = (warp - 3) >> 3, d = (warp - 3) & 7;
        const int hf = d / kSubsPerStage;              // which stage of the chunk holds my rows
        const int lrow = 16 * (d % kSubsPerStage) + (lane >> 1);   // row inside that stage
        const int row = 16 * d + (lane >> 1), hh = lane & 1;
        int as = 0, wseq = 0;
        uint32_t aph = 0;
        bool ok = true;
        for (int t = pair; t < p.tiles_total && ok; t += npairs) {
            const int rt = t / p.tiles_n;
            const int64_t t16 = (int64_t)rt * 16 + 8 * rank + d;     // this warp's 16-row sub-tile
            const bool has_rec = t16 < p.n_tiles16;
            for (int c = 0; c < p.nch && ok; ++c, wseq += kWHalves) {
                const int wslot = (wseq + hf) % C::kWStages;
                const uint32_t wpar = (uint32_t)(((wseq + hf) / C::kWStages) & 1);
                const uint8_t *wst = smem + C::kWOff + wslot * kGemmWStage;
                const uint32_t *rec = reinterpret_cast<const uint32_t *>(smem + C::kROff + wslot * C::kRecStage) +
                                      (d % kSubsPerStage) * kGemmRecCap;
                // this warp's patch entries for its two quarters of the chunk
                // (k-blocks dg and dg+2): lane j holds entries j and 32+j of
                // each, read from the staged record once the chunk has landed
                int qlo[2] = {0, 0}, qn[2] = {0, 0};
                uint32_t qe[2][2] = {{0u, 0u}, {0u, 0u}};
                for (int kq = 0; kq < 4; ++kq) {
                    const bool mine = (kq & 1) == dg;
                    if (mine) {
                        int w = 1;
                        if (lane == 0) {
                            if (kq == dg) w = role_wait(&w_full[wslot], wpar, abort_flag);
                            w = w && role_wait(&a_empty[as], aph ^ 1u, abort_flag);
                        }
                        w = __shfl_sync(0xffffffffu, w, 0);
                        if (!w) { ok = false; break; }
                        if (kq == dg && has_rec) {
                            // quarter boundaries 0 | n_q0 | n_low | n_q012 | n_all
                            const uint32_t h0 = rec[kRecHdr], h1 = rec[kRecHdr + 1];
                            const int bq[5] = {0, (int)(h1 & 0xFFFFu), (int)(h0 & 0xFFFFu), (int)(h1 >> 16), (int)(h0 >> 16)};
#pragma unroll
                            for (int u = 0; u < 2; ++u) {
                                const int q = dg + 2 * u;
                                const int lo = q == 0 ? bq[0] : q == 1 ? bq[1] : q == 2 ? bq[2] : bq[3];
                                const int hi = q == 0 ? bq[1] : q == 1 ? bq[2] : q == 2 ? bq[3] : bq[4];
                                qlo[u] = lo;
                                qn[u] = hi - lo;
                                const int j0 = kRecHdrWords + lo + lane;
                                qe[u][0] = (lane < qn[u] && j0 < kGemmRecCap) ? rec[j0] : 0u;
                                qe[u][1] = (lane + 32 < qn[u] && j0 + 32 < kGemmRecCap) ? rec[j0 + 32] : 0u;
                            }
                        }
                        uint8_t *ast = smem + C::kAOff + as * C::kAStage;
                        {
                            // row `row`, columns 64*kq + 32*hh .. +31 of the chunk
                            uint32_t sm[8], dw[4];
                            load_group_sw(wst, sw_group_offsets((uint32_t)lrow, (uint32_t)(2 * kq + hh)), sm, dw);
                            const uint32_t e2 = has_rec ? emax_x2(rec_emax(rec, lane >> 1, 2 * kq + hh)) : 0u;
                            GroupPairs gp;
                            decode_pairs_from<0>(gp, sm, dw, e2);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t col = 32u * hh + 8u * i;
                                *reinterpret_cast<uint4 *>(ast + sw128_offset((uint32_t)row, col)) =
                                    make_uint4(gp.w[4 * i], gp.w[4 * i + 1], gp.w[4 * i + 2], gp.w[4 * i + 3]);
                            }
                        }
                        __syncwarp();
                        if (has_rec) {
                            // exact values of this sub-tile's patched weights in the k-block
                            const int u = kq == dg ? 0 : 1;
                            const int n = u ? qn[1] : qn[0], lo = u ? qlo[1] : qlo[0];
                            auto put = [&](uint32_t ent) {
                                uint32_t rr, cc;
                                frag_position(ent, rr, cc);
                                *reinterpret_cast<uint16_t *>(ast + sw128_offset(16u * d + rr, cc & 63u)) =
                                    (uint16_t)(ent >> 16);
                            };
                            const int cap = kGemmRecCap - kRecHdrWords - lo;   // entries staged in shared memory
                            if (lane < n && lane < cap) put(u ? qe[1][0] : qe[0][0]);
                            if (lane + 32 < n && lane + 32 < cap) put(u ? qe[1][1] : qe[0][1]);
                            if (n > 64 || cap < n) {
                                // past the staged words or past 64 entries: from global memory
                                const int32_t base = __ldg(p.ptile_off + t16 * p.nch + c);
                                for (int j = lane; j < n; j += 32)
                                    if (j >= 64 || j >= cap) put(__ldg(p.precs + base + kRecHdrWords + lo + j));
                            }
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            // the leader's own warps arrive locally; the peer's across the pair
                            mbar_arrive(rank == 0 ? &a_full[as] : &a_ready[as]);
                        }
                    }
                    if (++as == C::kAStages) { as = 0; aph ^= 1u; }
                }
                if (!ok) break;
                if (lane == 0) mbar_arrive(&w_empty[wslot]);
            }
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int qd = warp & 3;                       // TMEM lane quarter
        int ac = 0;
        uint32_t acph = 0;
        for (int t = pair; t < p.tiles_total; t += npairs) {
            if (!role_wait(&acc_full[ac], acph, abort_flag)) break;
            tc_fence_after();
            const int rt = t / p.tiles_n, nt = t % p.tiles_n;
            const int64_t row = (int64_t)rt * 2 * kGemmBM + (int64_t)rank * kGemmBM + 32 * qd + lane;
            const float bias = (p.bias && row < p.rows) ? bf16_bits_to_f32(__ldg(p.bias + row)) : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem_base + ((uint32_t)(32 * qd) << 16) + (uint32_t)(ac * BN + c0), v);
                if (row < p.rows) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int64_t n = (int64_t)nt * BN + c0 + i;
                        if (n < p.M) {
                            const float o = __uint_as_float(v[i]) + bias;
                            if (p.y_f32) reinterpret_cast<float *>(p.y)[n * p.ldy + row] = o;
                            else reinterpret_cast<uint16_t *>(p.y)[n * p.ldy + row] = f32_to_bf16_bits_rn(o);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rank == 0) mbar_arrive(&acc_empty[ac]);
                else mbar_arrive_cluster(leader(&acc_empty[ac]));
            }
            if (++ac == C::kAccBufs) { ac = 0; acph ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    // neither CTA leaves (or frees tensor memory) while the other may still
    // signal its barriers or read its operands
    cluster_sync_all();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem_base), "r"(C::kTmemCols) : "memory");
    }
}


// ------------------------------------------------ slab kernel (large M)
// For many tokens the weight is decoded ONCE per 256-row slab instead of once
// per token tile: the pairs that first need a slab decode it (their share of
// its 16-row tiles, chunk by chunk) into a ring of bf16 slabs in global
// memory, small enough to stay in L2, and every token tile of the slab then
// streams it back with TMA, exactly like the activations.  The MMA pipeline
// is therefore a plain two-operand TMA pipeline (one barrier per stage, no
// per-k-block hand-off between decoder warps and the MMA issuer), and the
// decode work per flop drops by the number of token tiles per slab.
//
// Synchronisation between CTAs goes through two counters per (slab slot,
// chunk position) in the workspace, both monotonic within a launch:
//   ready   -- 16-row tiles decoded into that position (a slab's chunk is
//              readable once all of its tiles are in);
//   release -- token tiles that have finished loading that position (it may
//              be overwritten once every token tile of its slab is done).
// A slot holds a window of `wring` chunks of its slab; chunk c lives at
// position c % wring.  Every wait is bounded and raises the abort flag and
// the timeout status instead of hanging.  Each pair's decoder warps run
// through the pair's tiles in order (slab indices only grow) independently
// of its MMA, and a slot is reused only after slabs that lie about two
// rounds of pairs earlier (the ring has at least 2 * pairs / tiles-per-slab
// slots), so by induction on the slab index every wait ends when all CTAs
// are resident (the grid never exceeds the clusters that fit at once).
//
// NH = 256-token halves per tile.  NH = 1: tiles of 256 rows x 256 tokens,
// two accumulators in tensor memory (the epilogue of one tile overlaps the
// next tile's MMAs).  NH = 2: tiles of 256 rows x 512 tokens, each staged
// slab k-block feeding two N=256 MMAs (a quarter less L2 traffic per flop);
// the one 512-column accumulator is handed back to the MMA issuer in two
// halves, so the next tile's first MMAs only wait for the first half of the
// epilogue.
template <int NH>
struct SlabCfg {
    static constexpr int kStages = NH == 1 ? 6 : 4;
    static constexpr int kAStage = 128 * 128;       // 16 KB: 128 rows x 64 columns of the slab
    static constexpr int kBHalf = 128 * 128;        // 16 KB: this CTA's 128 tokens of a half x 64 columns
    static constexpr int kBStage = NH * kBHalf;
    static constexpr int kStage = kAStage + kBStage;
    // Warp roles, by warp index (a warp runs on sub-partition index % 4):
    // the MMA issuer shares its sub-partition only with the epilogue warp
    // of its TMEM lane quarter and two idle warps, away from the decoders.
    //   0 producer, 1 gate, 3 MMA issuer, 4..7 epilogue (lane quarter = index % 4),
    //   2, 8, 9, 10, 12, 13, 14 decoders, 11 and 15 idle.
    static constexpr int kWarps = 16;
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kDecWarps = 7;
    static constexpr int kProducerWarp = 0, kGateWarp = 1, kMmaWarp = 3, kFirstEpi = 4;
    __host__ __device__ static constexpr int dec_index(int w) {
        return w == 2 ? 0 : (w >= 8 && w <= 10) ? w - 7 : (w >= 12 && w <= 14) ? w - 8 : -1;
    }
    static constexpr int kGates = 8;                // chunks the gate may run ahead of the producer
    static constexpr int kBarOff = kStages * kStage;
    static constexpr int kNumBars = 2 * kStages + 4 + 2 * kGates;
    static constexpr int kMiscOff = kBarOff + kNumBars * 8;
    static constexpr int kSmem = kMiscOff + 16 + 1024;
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct SlabParams {
    CUtensorMap amap;          // slab ring [nslot * 256 rows][wring * 256] bf16, box 64 x 128, 128B swizzle
    CUtensorMap xmap;          // activations [M][in_f] bf16, box 64 x 128, 128B swizzle
    const uint8_t *layout;
    const int32_t *ptile_off;
    const uint32_t *precs;
    int64_t rows, M, row_bytes;
    int nch, n_tiles16, tiles_n, tiles_total, npairs;
    int nslot, wring;
    uint16_t *ring;            // [nslot][256][wring * 256]
    uint32_t *ready;           // [nslot][wring]
    uint32_t *release;         // [nslot][wring]
    const uint16_t *bias;
    void *y;
    int y_f32;
    int64_t ldy;
};

// load_group for the compressed weight in global memory, read once per
// launch: evict-first loads, so the stream of compressed weights does not
// push the decoded slabs and the activations (re-read by every tile) out of
// L2.
__device__ __forceinline__ void load_group_stream(const uint8_t *chunk, int q, uint32_t (&sm)[8], uint32_t (&dw)[4]) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4 *>(chunk + kSmOff + 32 * q));
    const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(chunk + kSmOff + 32 * q + 16));
    const uint4 d = __ldcs(reinterpret_cast<const uint4 *>(chunk + kDOff + 16 * q));
    sm[0] = a.x; sm[1] = a.y; sm[2] = a.z; sm[3] = a.w;
    sm[4] = b.x; sm[5] = b.y; sm[6] = b.z; sm[7] = b.w;
    dw[0] = d.x; dw[1] = d.y; dw[2] = d.z; dw[3] = d.w;
}

// Slab geometry shared by all roles.
struct SlabTile {
    int rt, nt;          // slab (256-row group) and token tile
    int slot, gen;       // ring slot and how many earlier slabs used it
    int n16;             // 16-row tiles in the slab
};

__device__ __forceinline__ SlabTile slab_tile(const SlabParams &p, int t) {
    SlabTile s;
    s.rt = t / p.tiles_n;
    s.nt = t - s.rt * p.tiles_n;
    s.slot = s.rt % p.nslot;
    s.gen = s.rt / p.nslot;
    s.n16 = min(16, p.n_tiles16 - 16 * s.rt);
    return s;
}

// Earlier uses of the ring position of chunk c by this slot (all slabs of
// earlier generations, then earlier laps of this slab), and the ready count
// at which chunk c of this slab is complete: earlier slabs are whole (16
// tiles; only the last slab can be shorter, and it is the last one to use
// its slot), this slab's laps up to and including c hold n16 tiles each.
__device__ __forceinline__ uint32_t slab_prior_uses(const SlabParams &p, const SlabTile &s, int c) {
    const int pos = c % p.wring;
    const int per_slab = (p.nch - 1 - pos) / p.wring + 1;
    return (uint32_t)(s.gen * per_slab + c / p.wring);
}

__device__ __forceinline__ uint32_t slab_ready_target(const SlabParams &p, const SlabTile &s, int c) {
    const int pos = c % p.wring;
    const int per_slab = (p.nch - 1 - pos) / p.wring + 1;
    return (uint32_t)(s.gen * per_slab * 16 + (c / p.wring + 1) * s.n16);
}

// The 16-row tiles [a, b) of its slab that token tile t decodes: every
// token tile of a slab decodes an equal share of its 16-row tiles, so the
// decode work is the same for every tile whatever the wave it falls in.
__device__ __forceinline__ void slab_share(const SlabParams &p, int t, int &a, int &b) {
    const int rt = t / p.tiles_n, j = t - rt * p.tiles_n;
    const int n16 = min(16, p.n_tiles16 - 16 * rt);
    a = n16 * j / p.tiles_n;
    b = n16 * (j + 1) / p.tiles_n;
}

template <int NH>
__global__ void __launch_bounds__(SlabCfg<NH>::kThreads, 1) gemm_slab_kernel(const __grid_constant__ SlabParams p) {
    using C = SlabCfg<NH>;
    constexpr int BN = 256 * NH;                   // tokens per tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
    uint64_t *full = bars, *empty = bars + C::kStages;
    uint64_t *acc_full = bars + 2 * C::kStages, *acc_empty = acc_full + 2;
    uint64_t *gate_full = acc_empty + 2, *gate_free = gate_full + C::kGates;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kMiscOff + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = (int)(blockIdx.x >> 1);
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int g = 0; g < C::kGates; ++g) { mbar_init(&gate_full[g], 1); mbar_init(&gate_free[g], 1); }
        // acc_empty: the 4 epilogue warps of each CTA
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 8); }
        abort_flag[0] = 0;
        fence_mbar_init();
    }
    cluster_sync_all();
    if (warp == C::kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(512) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    auto leader = [&](uint64_t *bar) { return mapa_shared(smem_u32(bar), 0u); };
    const uint32_t tmem_base = *tmem_slot;
    const int nkb = p.nch * 4;

    if (warp == C::kProducerWarp) {
        // ------------------------------------------------------- producer
        if (lane == 0) {
            prefetch_tensormap(&p.amap);
            prefetch_tensormap(&p.xmap);
            int s = 0, g = 0;
            uint32_t ph = 0, gph = 0;
            bool ok = true;
            for (int t = pair; t < p.tiles_total && ok; t += p.npairs) {
                const SlabTile st = slab_tile(p, t);
                for (int kb = 0; kb < nkb && ok; ++kb) {
                    const int c = kb >> 2, pos = c % p.wring;
                    if ((kb & 3) == 0) {
                        // this chunk of the slab decoded by every CTA that shares
                        // it: the gate warp has seen its ready count
                        if (!role_wait(&gate_full[g], gph, abort_flag)) { ok = false; break; }
                        fence_proxy_async_global();
                        mbar_arrive(&gate_free[g]);
                        if (++g == C::kGates) { g = 0; gph ^= 1u; }
                    }
                    if (!role_wait(&empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
                    const uint32_t lb = leader(&full[s]);
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * C::kStage));
                    uint8_t *stg = smem + s * C::kStage;
tma_load_2d_pair(stg, &p.amap, pos * kChunkElems + (kb & 3) * kGemmBK,
                                     st.slot * 256 + (int)rank * 128, lb);
#pragma unroll
                    for (int j = 0; j < NH; ++j)
                        tma_load_2d_pair(stg + C::kAStage + j * C::kBHalf, &p.xmap, kb * kGemmBK,
                                         st.nt * BN + 256 * j + (int)rank * 128, lb);
                    if (++s == C::kStages) { s = 0; ph ^= 1u; }
                }
            }
        }
    } else if (warp == C::kMmaWarp) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16_m<256, 256>();
            int s = 0, ac = 0;
            uint32_t ph = 0, acph = 0;
            bool ok = true;
            for (int t = pair; t < p.tiles_total && ok; t += p.npairs) {
                const SlabTile st = slab_tile(p, t);
                if constexpr (NH == 1) {
                    if (!role_wait(&acc_empty[ac], acph ^ 1u, abort_flag)) break;
                    tc_fence_after();
                }
                const uint32_t d_tmem = tmem_base + (uint32_t)(ac * 256);
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!role_wait(&full[s], ph, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    if ((kb & 3) == 3 || kb == nkb - 1) {
                        // both CTAs' copies of this chunk have landed: the pair no
                        // longer reads its ring position
                        atomicAdd(p.release + st.slot * p.wring + (kb >> 2) % p.wring, 1u);
                    }
                    const uint8_t *stg = smem + s * C::kStage;
                    const uint64_t ad = umma_desc_sw128(smem_u32(stg));
#pragma unroll
                    for (int j = 0; j < NH; ++j) {
                        if (NH == 2 && kb == 0) {
                            // the epilogue has drained this half of the accumulator
                            if (!role_wait(&acc_empty[j], acph ^ 1u, abort_flag)) { ok = false; break; }
                            tc_fence_after();
                        }
                        const uint64_t bd = umma_desc_sw128(smem_u32(stg + C::kAStage + j * C::kBHalf));
#pragma unroll
                        for (int k16 = 0; k16 < kGemmBK / 16; ++k16)
                            umma_bf16_pair(d_tmem + 256u * j, ad + 2u * k16, bd + 2u * k16, idesc, (kb | k16) != 0);
                    }
                    if (!ok) break;
                    umma_commit_pair_both(&empty[s]);
                    if (++s == C::kStages) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit_pair_both(&acc_full[ac]);
                if (NH == 1) {
                    if (++ac == 2) { ac = 0; acph ^= 1u; }
                } else {
                    acph ^= 1u;
                }
            }
        }
    } else if (warp == C::kGateWarp) {
        // ------------------------------------------------------- gate
        // Polls the ready counters of the producer's coming chunks (a
        // global acquire load takes about a microsecond) and passes each
        // on through a local barrier, so the producer never waits on L2.
        if (lane == 0) {
            int g = 0;
            uint32_t gph = 0;
            bool ok = true;
            for (int t = pair; t < p.tiles_total && ok; t += p.npairs) {
                const SlabTile st = slab_tile(p, t);
                for (int c = 0; c < p.nch; ++c) {
                    if (!role_wait(&gate_free[g], gph ^ 1u, abort_flag) ||
                        !counter_wait(p.ready + st.slot * p.wring + c % p.wring, slab_ready_target(p, st, c), abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive(&gate_full[g]);
                    if (++g == C::kGates) { g = 0; gph ^= 1u; }
                }
            }
        }
    } else if (warp >= C::kFirstEpi && warp < C::kFirstEpi + 4) {
        // ------------------------------------------------------- epilogue
        const int qd = warp & 3;                       // TMEM lane quarter
        int ac = 0;
        uint32_t acph = 0;
        for (int t = pair; t < p.tiles_total; t += p.npairs) {
            if (!role_wait(&acc_full[ac], acph, abort_flag)) break;
            tc_fence_after();
            const SlabTile st = slab_tile(p, t);
            const int64_t row = (int64_t)st.rt * 256 + (int64_t)rank * 128 + 32 * qd + lane;
            const float bias = (p.bias && row < p.rows) ? bf16_bits_to_f32(__ldg(p.bias + row)) : 0.f;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem_base + ((uint32_t)(32 * qd) << 16) + (uint32_t)(ac * 256 + c0), v);
                if (NH == 2 && c0 == 256 - 16) {
                    // first half drained: hand it back to the MMA issuer
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if (rank == 0) mbar_arrive(&acc_empty[0]);
                        else mbar_arrive_cluster(leader(&acc_empty[0]));
                    }
                }
                if (row < p.rows) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int64_t n = (int64_t)st.nt * BN + c0 + i;
                        if (n < p.M) {
                            const float o = __uint_as_float(v[i]) + bias;
if (p.y_f32) reinterpret_cast<float *>(p.y)[n * p.ldy + row] = o;
                            else reinterpret_cast<uint16_t *>(p.y)[n * p.ldy + row] = f32_to_bf16_bits_rn(o);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                uint64_t *bar = &acc_empty[NH == 1 ? ac : 1];
                if (rank == 0) mbar_arrive(bar);
                else mbar_arrive_cluster(leader(bar));
            }
            if (NH == 1) {
                if (++ac == 2) { ac = 0; acph ^= 1u; }
            } else {
                acph ^= 1u;
            }
        }
    } else if (C::dec_index(warp) >= 0) {
        // ------------------------------------------------------- decoders
        // An item is one 16-row tile x one chunk: lane (q = lane & 7, r =
        // lane >> 3) decodes group q (32 columns) of rows r, r+4, r+8, r+12
        // and stores them as bf16 into the slab ring; the item's patch
        // entries are then written over their saturated values.
        const int dw = C::dec_index(warp);
        const int q = lane & 7, r0 = lane >> 3;
        const int64_t ld = (int64_t)p.wring * kChunkElems;
        bool ok = true;
        for (int t = pair; t < p.tiles_total && ok; t += p.npairs) {
            int a, b;
            slab_share(p, t, a, b);
            const int ra = a + (b - a) * (int)rank / 2, rb = a + (b - a) * ((int)rank + 1) / 2;
            const int nr = rb - ra;
            if (nr <= 0) continue;
            const SlabTile st = slab_tile(p, t);
            const uint32_t tn = (uint32_t)p.tiles_n;
            for (int i = dw; i < p.nch * nr; i += C::kDecWarps) {
                const int c = i / nr, rtile = ra + (i - c * nr);
                const int pos = c % p.wring;
                const uint32_t prior = slab_prior_uses(p, st, c);
                if (prior > 0) {
                    // every token tile of the position's previous content is done with it
                    int w = 1;
                    if (lane == 0) w = counter_wait(p.release + st.slot * p.wring + pos, prior * tn, abort_flag);
                    if (!__shfl_sync(0xffffffffu, w, 0)) { ok = false; break; }
                }
                const int64_t t16 = (int64_t)st.rt * 16 + rtile;
                uint16_t *dst = p.ring + ((int64_t)st.slot * 256 + rtile * 16) * ld + (int64_t)pos * kChunkElems;
                // the record's offset first: its header load then overlaps the data's
                const bool has_rec = t16 < p.n_tiles16;
                const int32_t roff = has_rec ? __ldg(p.ptile_off + t16 * p.nch + c) : 0;
                uint32_t sm[4][8], dd[4][4], e2[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int64_t row = t16 * 16 + r0 + 4 * k;
                    if (row < p.rows) {
                        load_group_stream(p.layout + row * p.row_bytes + (int64_t)c * kChunkBytes, q, sm[k], dd[k]);
                        e2[k] = emax_x2(__ldg(reinterpret_cast<const uint8_t *>(p.precs + roff) + 8 * (r0 + 4 * k) + q));
                    } else {
#pragma unroll
                        for (int u = 0; u < 8; ++u) sm[k][u] = 0u;
                        dd[k][0] = dd[k][1] = dd[k][2] = dd[k][3] = 0u;
                        e2[k] = 0u;
                    }
                }
                const int n_all = has_rec ? (int)(__ldg(p.precs + roff + kRecHdr) >> 16) : 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    GroupPairs gp;
                    decode_pairs_from<0>(gp, sm[k], dd[k], e2[k]);
                    uint4 *o = reinterpret_cast<uint4 *>(dst + (int64_t)(r0 + 4 * k) * ld + 32 * q);
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        o[u] = make_uint4(gp.w[4 * u], gp.w[4 * u + 1], gp.w[4 * u + 2], gp.w[4 * u + 3]);
                }
                __syncwarp();
                if (has_rec) {
                    for (int j = lane; j < n_all; j += 32) {
                        const uint32_t ent = __ldcs(p.precs + roff + kRecHdrWords + j);
                        uint32_t rr, cc;
                        frag_position(ent, rr, cc);
                        dst[(int64_t)rr * ld + cc] = (uint16_t)(ent >> 16);
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    // the item's stores before the count, for the other CTAs'
                    // copy engines
                    fence_proxy_async_global();
                    __threadfence();
                    atomicAdd(p.ready + st.slot * p.wring + pos, 1u);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == C::kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(512) : "memory");
    }
}

static int gemm_sms() {
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

template <int BN>
static int launch_gemm(GemmParams &p, const uint8_t *layout, int64_t in_f, const uint16_t *x, int64_t ldx,
                       cudaStream_t st) {
    using C = GemmCfg<BN>;
    if (!encode_resident_map(&p.wmap, layout, p.rows, p.nch, resident_row_bytes(in_f), kGemmWRows))
        return set_error(BF16X_ERR_CUDA, "bf16x_gemm: weight tensor map");
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t xdims[2] = {(cuuint64_t)in_f, (cuuint64_t)p.M};
    const cuuint64_t xstr[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t xbox[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)BN};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), xdims, xstr, xbox, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return set_error(BF16X_ERR_CUDA, "bf16x_gemm: activation tensor map");
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64] = {false};
    if (dev < 0 || dev >= 64) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemm: device index");
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: smem attribute: %s", cudaGetErrorString(e));
        attr_set[dev] = true;
    }
    const int grid = std::min(p.tiles_total, gemm_sms());
    gemm_kernel<BN><<<grid, kGemmThreads, C::kSmem, st>>>(p);
    return check_launch("bf16x_gemm");
}

// CTA-pair launch: tiles of 256 rows x 256 tokens, clusters of 2 CTAs.
template <int BN>
static int launch_gemm2sm(GemmParams &p, const uint8_t *layout, int64_t in_f, const uint16_t *x, int64_t ldx,
                          cudaStream_t st) {
    using C = Gemm2Cfg<BN>;
    if (!encode_resident_map(&p.wmap, layout, p.rows, p.nch, resident_row_bytes(in_f), kGemmWRows))
        return set_error(BF16X_ERR_CUDA, "bf16x_gemm: weight tensor map");
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint64_t xdims[2] = {(cuuint64_t)in_f, (cuuint64_t)p.M};
    const cuuint64_t xstr[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t xbox[2] = {(cuuint32_t)kGemmBK, 128u};      // 128 tokens per copy (one or two per stage)
    const cuuint32_t estr[2] = {1, 1};
    if (fn(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), xdims, xstr, xbox, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return set_error(BF16X_ERR_CUDA, "bf16x_gemm: activation tensor map");
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64] = {false};
    if (dev < 0 || dev >= 64) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemm: device index");
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm2sm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: smem attribute: %s", cudaGetErrorString(e));
        attr_set[dev] = true;
    }
    const int pairs = std::max(1, std::min(p.tiles_total, gemm_sms() / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs));
    cfg.blockDim = dim3((unsigned)kGemmThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm2sm_kernel<BN>, p);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: pair launch: %s", cudaGetErrorString(e));
    return check_launch("bf16x_gemm");
}

// Slab-ring plan for a launch: used when every 256-row slab has at least 4
// token tiles and the tiles fill every pair at least once.  The ring holds
// the slabs of about two rounds of pairs, each as a window of at most the
// whole K, so that it stays well inside L2.
struct SlabPlan {
    bool use;
    int nh;                                         // 256-token halves per tile (1 or 2)
    int npairs, tiles_n, tiles_total, nslot, wring;
    int64_t ring_bytes, counter_bytes;
};

#ifndef BF16X_SLAB_RING_MB
#define BF16X_SLAB_RING_MB 64
#endif
constexpr int64_t kSlabRingMax = (int64_t)BF16X_SLAB_RING_MB << 20;

#ifndef BF16X_SLAB_WIDE
#define BF16X_SLAB_WIDE 1
#endif
static SlabPlan plan_slab(int64_t rows, int64_t in_f, int64_t M, int sms) {
    SlabPlan s = {};
    const int64_t nch = (in_f + kChunkElems - 1) / kChunkElems;
    const int64_t tiles_m2 = (rows + 255) / 256;
    s.npairs = std::max(1, sms / 2);
    // 512-token tiles move a quarter less data per flop but expose half an
    // epilogue per tile; measured, they pay for long K only (K >= 8192), and
    // then only when their last round of pairs is not much emptier than with
    // 256-token tiles (wave efficiency x 1.15 against wave efficiency)
    auto wave_eff = [&](int64_t tiles) {
        return (double)tiles / (double)(((tiles + s.npairs - 1) / s.npairs) * s.npairs);
    };
    const int64_t tn1 = (M + 255) / 256, tn2 = (M + 511) / 512;
#ifndef BF16X_SLAB_MIN_TN
#define BF16X_SLAB_MIN_TN 4
#endif
    const bool ok1 = tn1 >= BF16X_SLAB_MIN_TN && tiles_m2 * tn1 >= s.npairs;
    const bool ok2 = BF16X_SLAB_WIDE && nch >= 32 && tn2 >= 2 && tiles_m2 * tn2 >= s.npairs;
    if (!ok1 && !ok2) return s;
    s.nh = (ok2 && (!ok1 || 1.15 * wave_eff(tiles_m2 * tn2) >= wave_eff(tiles_m2 * tn1))) ? 2 : 1;
    const int64_t tn = s.nh == 2 ? tn2 : tn1;
    if (tiles_m2 * tn > 0x7fffffffLL) return s;
    s.tiles_n = (int)tn;
    s.tiles_total = (int)(tiles_m2 * tn);
#ifndef BF16X_SLAB_SLACK
#define BF16X_SLAB_SLACK 1
#endif
    s.nslot = (int)std::min<int64_t>(tiles_m2, BF16X_SLAB_SLACK * ((2 * s.npairs + tn - 1) / tn) + 2);
    const int64_t slab_chunk_bytes = 256ll * kChunkElems * 2;      // one chunk of one slab
    s.wring = (int)std::min<int64_t>(nch, std::max<int64_t>(4, kSlabRingMax / (s.nslot * slab_chunk_bytes)));
    s.ring_bytes = (int64_t)s.nslot * s.wring * slab_chunk_bytes;
    s.counter_bytes = ((int64_t)2 * s.nslot * s.wring * 4 + 255) / 256 * 256;
    s.use = true;
    return s;
}

static int launch_gemm_slab(const SlabPlan &pl, const uint8_t *layout, const int32_t *ptile_off,
                            const uint32_t *precs, int64_t rows, int64_t in_f, const uint16_t *x, int64_t M,
                            int64_t ldx, const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *ws,
                            cudaStream_t st) {
    SlabParams p;
    p.layout = layout;
    p.ptile_off = ptile_off;
    p.precs = precs;
    p.rows = rows;
    p.M = M;
    p.row_bytes = resident_row_bytes(in_f);
    p.nch = (int)((in_f + kChunkElems - 1) / kChunkElems);
    p.n_tiles16 = (int)((rows + kTileRows - 1) / kTileRows);
    p.tiles_n = pl.tiles_n;
    p.tiles_total = pl.tiles_total;
    p.npairs = std::min(pl.npairs, pl.tiles_total);
    p.nslot = pl.nslot;
    p.wring = pl.wring;
    uint8_t *base = static_cast<uint8_t *>(ws);
    p.ready = reinterpret_cast<uint32_t *>(base);
    p.release = p.ready + (int64_t)pl.nslot * pl.wring;
    p.ring = reinterpret_cast<uint16_t *>(base + pl.counter_bytes);
    p.bias = bias;
    p.y = y;
    p.y_f32 = y_dtype == BF16X_DTYPE_F32;
    p.ldy = ldy;
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: cuTensorMapEncodeTiled unavailable");
    const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, 128u};
    const cuuint32_t estr[2] = {1, 1};
    const cuuint64_t adims[2] = {(cuuint64_t)pl.wring * kChunkElems, (cuuint64_t)pl.nslot * 256};
    const cuuint64_t astr[1] = {(cuuint64_t)pl.wring * kChunkElems * 2};
    if (fn(&p.amap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.ring, adims, astr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return set_error(BF16X_ERR_CUDA, "bf16x_gemm: slab tensor map");
    const cuuint64_t xdims[2] = {(cuuint64_t)in_f, (cuuint64_t)M};
    const cuuint64_t xstr[1] = {(cuuint64_t)ldx * 2};
    if (fn(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t *>(x), xdims, xstr, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return set_error(BF16X_ERR_CUDA, "bf16x_gemm: activation tensor map");
    // counters start at zero in every launch
    cudaError_t e = cudaMemsetAsync(base, 0, (size_t)pl.counter_bytes, st);
    void (*kern)(SlabParams) = pl.nh == 2 ? gemm_slab_kernel<2> : gemm_slab_kernel<1>;
    const int smem_bytes = pl.nh == 2 ? SlabCfg<2>::kSmem : SlabCfg<1>::kSmem;
    const int threads = SlabCfg<1>::kThreads;
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: clearing counters: %s", cudaGetErrorString(e));
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr_set[64][2] = {};
    if (dev < 0 || dev >= 64) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemm: device index");
    const int vi = pl.nh - 1;
    if (!attr_set[dev][vi]) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
        if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: smem attribute: %s", cudaGetErrorString(e));
        attr_set[dev][vi] = true;
    }
    // the CTAs wait on one another's progress, so every pair must be resident
    // at once: no more pairs than clusters of 2 that fit on the device
    static int max_clusters[64][2] = {};
    if (!max_clusters[dev][vi]) {
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3((unsigned)(2 * pl.npairs));
        q.blockDim = dim3((unsigned)threads);
        q.dynamicSmemBytes = smem_bytes;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = 2;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        q.attrs = qa;
        q.numAttrs = 1;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, kern, &q);
        if (e != cudaSuccess || n < 1)
            return set_error(BF16X_ERR_CUDA, "bf16x_gemm: cluster occupancy: %s", cudaGetErrorString(e));
        max_clusters[dev][vi] = n;
    }
    p.npairs = std::min(p.npairs, max_clusters[dev][vi]);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * p.npairs));
    cfg.blockDim = dim3((unsigned)threads);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) return set_error(BF16X_ERR_CUDA, "bf16x_gemm: slab launch: %s", cudaGetErrorString(e));
    return check_launch("bf16x_gemm");
}

}  // namespace bf16x

using namespace bf16x;

extern "C" int64_t bf16x_gemm_workspace_bytes(int64_t rows, int64_t in_f, int64_t M) {
    if (rows <= 0 || in_f <= 0 || M <= 0 || in_f > 65536) return 0;
    const SlabPlan pl = plan_slab(rows, in_f, M, gemm_sms());
    return pl.use ? pl.counter_bytes + pl.ring_bytes : 0;
}

extern "C" int bf16x_gemm_ws(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                             int64_t rows, int64_t in_f, const uint16_t *x, int64_t M, int64_t ldx,
                             const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *workspace,
                             int64_t workspace_bytes, void *stream) {
    if (rows < 0 || in_f <= 0 || M < 0) return set_error(BF16X_ERR_INVALID, "bf16x_gemm: bad shape");
    if (in_f > 65536) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemm: in_f > 65536");
    if (y_dtype != BF16X_DTYPE_BF16 && y_dtype != BF16X_DTYPE_F32)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemm: bad y_dtype");
    if (rows == 0 || M == 0) return BF16X_OK;
    if (!layout || !ptile_off || !precs || !x || !y) return set_error(BF16X_ERR_INVALID, "bf16x_gemm: null pointer");
    if (ldx < in_f || (ldx % 8) != 0) return set_error(BF16X_ERR_INVALID, "bf16x_gemm: ldx must be >= in_f and a multiple of 8");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(layout) | reinterpret_cast<uintptr_t>(precs)) & 15u)
        return set_error(BF16X_ERR_INVALID, "bf16x_gemm: x, layout and records must be 16-byte aligned");
    if (ldy < rows) return set_error(BF16X_ERR_INVALID, "bf16x_gemm: ldy < rows");
    GemmParams p;
    p.ptile_off = ptile_off;
    p.precs = precs;
    p.rows = rows;
    p.M = M;
    p.nch = (int)((in_f + kChunkElems - 1) / kChunkElems);
    p.n_tiles16 = (int)((rows + kTileRows - 1) / kTileRows);
    p.bias = bias;
    p.y = y;
    p.y_f32 = y_dtype == BF16X_DTYPE_F32;
    p.ldy = ldy;
    const int64_t tiles_m = (rows + kGemmBM - 1) / kGemmBM;
    cudaStream_t st = (cudaStream_t)stream;
    const int sms = gemm_sms();
    if (workspace) {
        const SlabPlan pl = plan_slab(rows, in_f, M, sms);
        if (pl.use) {
            if (workspace_bytes < pl.counter_bytes + pl.ring_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u))
                return set_error(BF16X_ERR_INVALID, "bf16x_gemm: workspace of %lld bytes (256-byte aligned) needed",
                                 (long long)(pl.counter_bytes + pl.ring_bytes));
            return launch_gemm_slab(pl, layout, ptile_off, precs, rows, in_f, x, M, ldx, bias, y, y_dtype, ldy,
                                    workspace, st);
        }
    }
    // token tile: 256 when that still fills the GPU, else smaller
    int bn = M <= 64 ? 64 : M <= 128 ? 128 : 256;
    if (bn == 256 && tiles_m * ((M + 255) / 256) < sms) bn = 128;
#ifndef BF16X_GEMM_NO_PAIR
    if (bn == 256) {
        // CTA pairs: tiles of 256 rows x 256 tokens, or x 512 tokens when
        // that is one tile per 256-row slab and the slabs fit in one round of
        // pairs: each weight is then decoded once.  With more rounds the
        // shallower rings and the single accumulator (no epilogue overlap)
        // of 512-token tiles cost more than the halved decode saves.
        const int64_t slabs = (rows + 2 * kGemmBM - 1) / (2 * kGemmBM);
        const int pbn = (M > 256 && M <= 512 && slabs <= sms / 2) ? 512 : 256;
        p.tiles_n = (int)((M + pbn - 1) / pbn);
        const int64_t total2 = (rows + 2 * kGemmBM - 1) / (2 * kGemmBM) * p.tiles_n;
        if (total2 > 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemm: too many tiles");
        p.tiles_total = (int)total2;
        return pbn == 512 ? launch_gemm2sm<512>(p, layout, in_f, x, ldx, st)
                          : launch_gemm2sm<256>(p, layout, in_f, x, ldx, st);
    }
#endif
    p.tiles_n = (int)((M + bn - 1) / bn);
    const int64_t total = tiles_m * p.tiles_n;
    if (total > 0x7fffffffLL) return set_error(BF16X_ERR_UNSUPPORTED, "bf16x_gemm: too many tiles");
    p.tiles_total = (int)total;
    if (bn == 64) return launch_gemm<64>(p, layout, in_f, x, ldx, st);
    if (bn == 128) return launch_gemm<128>(p, layout, in_f, x, ldx, st);
    return launch_gemm<256>(p, layout, in_f, x, ldx, st);
}

extern "C" int bf16x_gemm(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                          int64_t rows, int64_t in_f, const uint16_t *x, int64_t M, int64_t ldx,
                          const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *stream) {
    return bf16x_gemm_ws(layout, ptile_off, precs, rows, in_f, x, M, ldx, bias, y, y_dtype, ldy, nullptr, 0, stream);
}
