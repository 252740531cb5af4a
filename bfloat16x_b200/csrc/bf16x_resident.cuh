// bf16x_resident.cuh -- the resident ("kernel") layout and its pair decoder.
//
// A weight of [rows][in_f] is stored row by row in chunks of 256 columns
// (in_f padded up to a multiple of 256).  One chunk is 368 bytes:
//
//   [  0, 256)  sign|mantissa byte per element, natural column order:
//               byte = sign << 7 | mant7
//   [256, 352)  deltas of 8 groups of 32 columns, 12 bytes (3 words) each:
//               pair p (columns 2p, 2p+1 of the group), p < 15, lives in word
//               p / 5 at slot s = p % 5: low delta at bits 3s..3s+2, high
//               delta at bits 16+3s..16+3s+2; pair 15 spreads its two 3-bit
//               deltas over bit 15 (low) and bit 31 (high) of the 3 words
//               (bit i of each delta in word i).  7 = saturated.
//   [352, 368)  emax of the 16 sub-blocks of 16 columns (row-local)
//
// That is exactly 11.5 bits per weight, the same as the flat streams, but
// laid out so that one pair of weights becomes one bf16x2 register in five
// integer operations (prmt, lop3, shf, lop, iadd):
//
//   x    = prmt(smword, 0, 0x1100 | 0x3322)   -> [b0 b0 b1 b1]
//   w    = (x & 0x807F807F) | emax * 0x00800080
//   w   -= (dword shifted so the two deltas sit at bits 7 and 23) & 0x03800380
//
// The subtraction never borrows across fields because delta <= emax.  Weights
// whose exact delta exceeds 7 decode to emax - 7 here and are corrected from
// the patch records.
//
// Patch records: rows are grouped in tiles of 16; for every (tile, chunk)
// there is one record of 16-byte-aligned words at precs + ptile_off[tile *
// nchunks + chunk]:
//   word 0       n_low (bits 0..15): entries in columns 0..127 of the chunk,
//                n_all (bits 16..31): all entries
//   word 1       n_q0 (bits 0..15): entries in columns 0..63,
//                n_q012 (bits 16..31): entries in columns 0..191
//   words 2..    entries grouped by 64-column quarter (in quarter order;
//                within a quarter dealt round-robin over the shared-memory
//                banks of their fragment words), u32 each:
//                frag (bits 0..10) | half (bit 11) | exact bf16 bits << 16
//                where half = column >= 128 and frag is the element's 16-bit
//                slot in the mma fragment order of its half chunk (see
//                frag_index): the GEMV stores the value there directly.
//   zero padding to a multiple of 4 words.
// ptile_off has n_tiles * nchunks + 1 entries; the last one is the total.
#pragma once

#include "bf16x_common.cuh"

namespace bf16x {

constexpr int kChunkElems = 256;
constexpr int kChunkBytes = 368;
constexpr int kSmOff = 0;
constexpr int kDOff = 256;
constexpr int kEOff = 352;
constexpr int kTileRows = 16;
constexpr int kRecHdrWords = 2;

__host__ __device__ inline int64_t rec_words(int64_t n_entries) {
    return (kRecHdrWords + n_entries + 3) / 4 * 4;
}

__host__ __device__ inline int64_t resident_row_bytes(int64_t in_f) {
    return (in_f + kChunkElems - 1) / kChunkElems * kChunkBytes;
}

// Delta field of pair P of a group (3 words), positioned at bits 7..9 / 23..25.
template <int P>
__device__ __forceinline__ uint32_t pair_delta(const uint32_t (&dw)[3]) {
    if constexpr (P < 15) {
        constexpr int W = P / 5, S = P % 5;
        return shl_signed<7 - 3 * S>(dw[W]) & 0x03800380u;
    } else {
        return ((dw[0] >> 8) & 0x00800080u) | ((dw[1] >> 7) & 0x01000100u) |
               ((dw[2] >> 6) & 0x02000200u);
    }
}

// bf16x2 bits of pair P of a group: sm = the group's 8 sign|mant words,
// e2 = emax * 0x00800080 of the pair's sub-block.
template <int P>
__device__ __forceinline__ uint32_t decode_pair(const uint32_t (&sm)[8], const uint32_t (&dw)[3], uint32_t e2) {
    constexpr uint32_t sel = (P & 1) ? 0x3322u : 0x1100u;
    const uint32_t x = prmt(sm[P >> 1], 0u, sel);
    return ((x & 0x807F807Fu) | e2) - pair_delta<P>(dw);
}

// Decode all 16 pairs of one 32-column group.
struct GroupPairs {
    uint32_t w[16];
};

template <int P>
__device__ __forceinline__ void decode_pairs_from(GroupPairs &g, const uint32_t (&sm)[8],
                                                  const uint32_t (&dw)[3], uint32_t e2lo, uint32_t e2hi) {
    g.w[P] = decode_pair<P>(sm, dw, P < 8 ? e2lo : e2hi);
    if constexpr (P + 1 < 16) decode_pairs_from<P + 1>(g, sm, dw, e2lo, e2hi);
}

// Load group q of a chunk (generic pointer: shared or global memory).
__device__ __forceinline__ void load_group(const uint8_t *chunk, int q, uint32_t (&sm)[8],
                                           uint32_t (&dw)[3], uint32_t &e2lo, uint32_t &e2hi) {
    const uint4 a = *reinterpret_cast<const uint4 *>(chunk + kSmOff + 32 * q);
    const uint4 b = *reinterpret_cast<const uint4 *>(chunk + kSmOff + 32 * q + 16);
    sm[0] = a.x; sm[1] = a.y; sm[2] = a.z; sm[3] = a.w;
    sm[4] = b.x; sm[5] = b.y; sm[6] = b.z; sm[7] = b.w;
    const uint32_t *d = reinterpret_cast<const uint32_t *>(chunk + kDOff + 12 * q);
    dw[0] = d[0]; dw[1] = d[1]; dw[2] = d[2];
    const uint32_t e = *reinterpret_cast<const uint16_t *>(chunk + kEOff + 2 * q);
    e2lo = (e & 0xFFu) * 0x00800080u;
    e2hi = (e >> 8) * 0x00800080u;
}

// Position of element (row, col) of a 16-row x 256-column chunk inside the
// mma.m16n8k16 A-fragment buffer of its half (128 columns): 8 steps x 32
// lanes x 4 registers x 2 halves of 16 bits.  Lane (g, t) holds rows g and
// g+8 of the 32-column group t; step J carries group columns 4J..4J+3 as
// pairs 2J (registers 0/1: rows g/g+8) and 2J+1 (registers 2/3).  The lane's
// 16 bytes of step J sit at slot J * 32 + (lane ^ J): a permutation within
// the step, so the fragment stores and loads stay conflict-free, that spreads
// the patch entries of a 64-column quarter over all 32 shared-memory banks.
__host__ __device__ inline uint32_t frag_index(uint32_t row, uint32_t col) {
    const uint32_t kk = col & 127u;
    const uint32_t owner = 4u * (row & 7u) + (kk >> 5);
    const uint32_t step = (kk >> 2) & 7u;
    const uint32_t reg = (row >> 3) + 2u * ((kk >> 1) & 1u);
    return (step * 32u + (owner ^ step)) * 8u + reg * 2u + (kk & 1u);
}

// Inverse of frag_index: (row, col) from a patch entry.
__host__ __device__ inline void frag_position(uint32_t entry, uint32_t &row, uint32_t &col) {
    const uint32_t idx = entry & 0x7FFu, half = (entry >> 11) & 1u;
    const uint32_t step = idx >> 8;
    const uint32_t hw = idx & 1u, reg = (idx >> 1) & 3u, owner = ((idx >> 3) & 31u) ^ step;
    row = (owner >> 2) + 8u * (reg & 1u);
    col = 128u * half + 32u * (owner & 3u) + 4u * step + 2u * (reg >> 1) + hw;
}

// Exact bf16 bits of a patched element (flat-entry form: delta, sign|mant).
__device__ __forceinline__ uint32_t patch_bits(uint32_t entry, uint32_t emax) {
    const uint32_t val = (entry >> 16) & 0xFFu, sm = entry >> 24;
    return ((sm & 0x80u) << 8) | (((emax - val) & 0xFFu) << 7) | (sm & 0x7Fu);
}

// The saturated (delta 7) bits the main decode produced for that element.
__device__ __forceinline__ uint32_t saturated_bits(uint32_t entry, uint32_t emax) {
    const uint32_t sm = entry >> 24;
    return ((sm & 0x80u) << 8) | (((emax - 7u) & 0xFFu) << 7) | (sm & 0x7Fu);
}

}  // namespace bf16x
