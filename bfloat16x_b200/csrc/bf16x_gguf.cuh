// bf16x_gguf.cuh -- GGUF BF16X blocks read in place by the fused GEMV.
//
// A GGUF BF16X weight (llama.cpp GGML_TYPE_BF16X, bf16x_gguf_block.py:1-20)
// is stored row by row as 46-byte blocks of 32 weights:
//
//   bytes  0..1   emax of weights 0..15 and 16..31 (floored at 7 by the packer)
//   bytes  2..5   32 sign bits, LSB-first
//   bytes  6..33  32 x 7-bit mantissas, LSB-first
//   bytes 34..45  32 x 3-bit exponent deltas, LSB-first; 7 = zero marker
//
// decoded (bf16x_gguf_block.py:84-95) as sign | e << 7 | mant with
// e = 0 for delta 7 and max(emax - delta, 0) otherwise.  With in_f a multiple
// of 256 one row-chunk of 256 columns is 8 blocks = 368 bytes, a multiple of
// 16, so a 16-row x 256-column item is one 2-D TMA box of the block array
// itself: the GEMV streams the 11.5 bits per weight of the file format.
//
// Every field starts on a 16-bit boundary of its block, and a block starts on
// a 16-bit boundary of shared memory, so a lane gathers the fields with
// byte permutes.  It decodes a block into 16 bf16x2 registers, register P
// holding weights P (low half) and P + 16 (high half): the two mantissa
// streams (weights 0..15 and 16..31) are interleaved halfword by halfword,
// after which one shift extracts both mantissas of a pair, and likewise for
// the deltas; the sign word shifted by 15 - P puts both signs of the pair in
// place.  The activations are permuted to the same pair order.
//
// The lossless side table ({u16 col, u16 bf16 bits} per clamped weight, by
// row, bf16x_gguf_block.py:107-161) is re-indexed once into one record per
// (16-row tile, 256-column chunk), like the resident layout's patch records:
//   word 0       n_low (bits 0..15): entries of half 0, n_all (16..31): all
//   words 1..3   zero
//   words 4..    entries, half 0 first, within a half by row then column:
//                frag (bits 0..10) | half (bit 11) | exact bf16 bits << 16
// where half = block index & 1 (the even blocks are decoded in the first
// half of the item, the odd ones in the second) and frag is the weight's
// 16-bit slot among that half's mma fragments (gguf_frag_index).  The GEMV
// stores the exact values over the decoded fragments.
#pragma once

#include "bf16x_common.cuh"

namespace bf16x {

constexpr int kGgufBlockBytes = 46;
constexpr int kGgufChunkBytes = 8 * kGgufBlockBytes;      // 368
constexpr int kGgufChunkWords = kGgufChunkBytes / 4;      // 92
constexpr int kGgufRecHdrWords = 4;

__host__ __device__ inline int64_t gguf_rec_words(int64_t n_entries) {
    return (kGgufRecHdrWords + n_entries + 3) / 4 * 4;
}

__host__ __device__ inline int64_t gguf_row_bytes(int64_t in_f) { return in_f / 32 * kGgufBlockBytes; }

// Slot of weight (row, col) of an item (row < 16, col < 256) among the mma
// fragments of its half: lane (g, t) decodes block 2t + half of rows g and
// g + 8; mma step J carries pairs 2J (registers 0/1: rows g / g+8) and
// 2J + 1 (registers 2/3); pair P is weights P and P + 16 of the block.  The
// index is (J * 32 + (lane ^ J)) * 8 + register * 2 + halfword, the layout of
// the GEMV's fragment buffer.
__host__ __device__ inline uint32_t gguf_frag_index(uint32_t row, uint32_t col) {
    const uint32_t q = (col >> 5) & 7u, t = q >> 1, jj = col & 31u, P = jj & 15u;
    const uint32_t step = P >> 1, reg = (row >> 3) + 2u * (P & 1u);
    const uint32_t owner = 4u * (row & 7u) + t;
    return (step * 32u + (owner ^ step)) * 8u + reg * 2u + (jj >> 4);
}

// Inverse of gguf_frag_index: (row, col) of a record entry.
__host__ __device__ inline void gguf_frag_position(uint32_t entry, uint32_t &row, uint32_t &col) {
    const uint32_t idx = entry & 0x7FFu, half = (entry >> 11) & 1u;
    const uint32_t step = idx >> 8, hw = idx & 1u, reg = (idx >> 1) & 3u;
    const uint32_t owner = ((idx >> 3) & 31u) ^ step;
    row = (owner >> 2) + 8u * (reg & 1u);
    col = 32u * (2u * (owner & 3u) + half) + 2u * step + (reg >> 1) + 16u * hw;
}

// lop3 / prmt with their constant operand as an immediate (no register to
// hold it across the unrolled decode)
template <uint32_t LUT, uint32_t C>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(r) : "r"(a), "r"(b), "n"(C), "n"(LUT));
    return r;
}
template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt_i(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "n"(SEL));
    return r;
}
// truth tables (A = 0xF0, B = 0xCC, C = 0xAA)
constexpr uint32_t kSelAC_BnC = 0xE4;   // (a & c) | (b & ~c)
constexpr uint32_t kSelAnC_BC = 0xD8;   // (a & ~c) | (b & c)
constexpr uint32_t kAC_or_B = 0xEC;     // (a & c) | b
constexpr uint32_t kAnB_CB = 0xB8;      // (a & ~b) | (c & b)

// Halfwords I (low) and J (high) of a 12-word window.
template <int I, int J>
__device__ __forceinline__ uint32_t gguf_hw2(const uint32_t (&w)[12]) {
    if constexpr ((I & 1) == 0 && J == I + 1) {
        return w[I >> 1];
    } else {
        constexpr uint32_t sel = (2u * (I & 1)) | ((2u * (I & 1) + 1u) << 4) | ((4u + 2u * (J & 1)) << 8) |
                                 ((5u + 2u * (J & 1)) << 12);
        return prmt_i<sel>(w[I >> 1], w[J >> 1]);
    }
}

// The fields of one block, the two 16-weight streams of mantissas and deltas
// interleaved halfword by halfword: z[k] = halfword k of the mantissas of
// weights 0..15 | that of weights 16..31 << 16, dz[k] the same for deltas.
struct GgufBlock {
    uint32_t z[7], dz[3];
    uint32_t zs[6], dzs[2];   // the same shifted by 8 bits: a field that crosses a halfword of z / dz lies inside one of these
    uint32_t sign;      // bit j = sign of weight j
    uint32_t e7;        // emax0 << 7 | emax1 << 23
    uint32_t emax;      // emax0 | emax1 << 8
    uint32_t c16;       // (emax0 - 7) | (emax1 - 7) << 16
};

// Block starting at halfword H (0 or 1) of the window.
template <int H>
__device__ __forceinline__ GgufBlock gguf_load_block(const uint32_t (&w)[12]) {
    GgufBlock b;
    b.sign = gguf_hw2<H + 1, H + 2>(w);
    b.z[0] = gguf_hw2<H + 3, H + 10>(w);
    b.z[1] = gguf_hw2<H + 4, H + 11>(w);
    b.z[2] = gguf_hw2<H + 5, H + 12>(w);
    b.z[3] = gguf_hw2<H + 6, H + 13>(w);
    b.z[4] = gguf_hw2<H + 7, H + 14>(w);
    b.z[5] = gguf_hw2<H + 8, H + 15>(w);
    b.z[6] = gguf_hw2<H + 9, H + 16>(w);
    b.dz[0] = gguf_hw2<H + 17, H + 20>(w);
    b.dz[1] = gguf_hw2<H + 18, H + 21>(w);
    b.dz[2] = gguf_hw2<H + 19, H + 22>(w);
#pragma unroll
    for (int k = 0; k < 6; ++k) b.zs[k] = prmt_i<0x6341u>(b.z[k], b.z[k + 1]);
#pragma unroll
    for (int k = 0; k < 2; ++k) b.dzs[k] = prmt_i<0x6341u>(b.dz[k], b.dz[k + 1]);
    // emax bytes to bytes 0 and 2 (byte 4 of the pair is the zero operand)
    constexpr uint32_t esel = (2u * H) | (4u << 4) | ((2u * H + 1u) << 8) | (4u << 12);
    b.e7 = prmt_i<esel>(w[0], 0u) << 7;
    b.emax = H ? (w[0] >> 16) : (w[0] & 0xFFFFu);
    b.c16 = prmt_i<esel>(w[0], 0u) - 0x00070007u;
    return b;
}

// Smallest emax of a block (both halves).
template <int H>
__device__ __forceinline__ uint32_t gguf_min_emax(const uint32_t (&w)[12]) {
    const uint32_t e = H ? (w[0] >> 16) : w[0];
    return min(e & 0xFFu, (e >> 8) & 0xFFu);
}

// bf16x2 bits of pair P (weights P and P + 16).  FAST requires emax >= 7 in
// both halves (the packer floors it at 7): with u = 7 - delta and
// c = emax - 7 per 16-bit half, the exponent min(u + c, 257 u) is 0 for the
// zero marker (u = 0) and emax - delta otherwise, one DPX add-min for both
// halves.  Otherwise each lane takes max(emax - delta, 0) on its own.
template <int P, bool FAST>
__device__ __forceinline__ uint32_t gguf_pair(const GgufBlock &b) {
    constexpr int mr = (7 * P) & 15, mk = (7 * P) >> 4;
    uint32_t m;
    if constexpr (mr <= 9) m = b.z[mk] >> mr;      // both mantissas at bits 0..6 / 16..22
    else m = b.zs[mk] >> (mr - 8);
    constexpr int dr = (3 * P) & 15, dk = (3 * P) >> 4;
    uint32_t v;
    if constexpr (FAST) {
        const uint32_t x = dr <= 13 ? b.dz[dk] >> dr : b.dzs[dk] >> (dr - 8);
        const uint32_t u = lop3<0x0A, 0x00070007u>(x, x);           // 7 - delta per half
        const uint32_t e = __viaddmin_u16x2(u, b.c16, u * 257u);   // 0 for the marker, else emax - delta
        v = e << 7;
    } else {
        uint32_t d;
        if constexpr (dr <= 13) {
            d = shl_signed<7 - dr>(b.dz[dk]);
        } else {
            constexpr uint32_t c = (dr == 14 ? 0x0200u : 0x0300u) * 0x10001u;
            d = lop3<kSelAnC_BC, c>(b.dz[dk] >> (dr - 7), b.dz[dk + 1] << (23 - dr));
        }
        d &= 0x03800380u;
        const uint32_t d0 = (d >> 7) & 7u, d1 = (d >> 23) & 7u;
        const uint32_t e0 = b.emax & 0xFFu, e1 = (b.emax >> 8) & 0xFFu;
        const uint32_t x0 = (d0 == 7u || d0 > e0) ? 0u : e0 - d0;
        const uint32_t x1 = (d1 == 7u || d1 > e1) ? 0u : e1 - d1;
        v = (x0 << 7) | (x1 << 23);
    }
    const uint32_t u = lop3<kSelAC_BnC, 0x007F007Fu>(m, b.sign << (15 - P));
    return lop3<kAC_or_B, 0x807F807Fu>(u, v);
}

template <int P, bool FAST>
__device__ __forceinline__ void gguf_pairs_from(const GgufBlock &b, uint32_t (&out)[16]) {
    out[P] = gguf_pair<P, FAST>(b);
    if constexpr (P + 1 < 16) gguf_pairs_from<P + 1, FAST>(b, out);
}

}  // namespace bf16x
