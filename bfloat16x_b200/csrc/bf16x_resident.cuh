// bf16x_resident.cuh -- the resident ("kernel") layout and its pair decoder.
//
// A weight of [rows][in_f] is stored row by row in chunks of 256 columns
// (in_f padded up to a multiple of 256).  One chunk is 384 bytes:
//
//   [  0, 256)  sign|mantissa byte per element, natural column order:
//               byte = sign << 7 | mant7
//   [256, 384)  4-bit exponent deltas of the 8 groups of 32 columns, 16
//               bytes (4 words) per group: pair p of a group (columns 2p,
//               2p+1) sits in word p / 4 at slot s = p % 4, low delta at bits
//               4s..4s+3, high delta at bits 16+4s..16+4s+3.  15 = saturated.
//
// Each group's shared exponent (emax, the largest exponent of its 32
// weights) lives in the patch record of the group's (16-row tile, chunk),
// below: 12 bits per weight in the chunk + 1/4 bit of emax.
//
// One pair of weights becomes one bf16x2 register in five integer
// operations (prmt, lop3, shf, lop, iadd):
//
//   x    = prmt(smword, 0, 0x1100 | 0x3322)   -> [b0 b0 b1 b1]
//   w    = (x & 0x807F807F) | emax * 0x00800080
//   w   -= (dword shifted so the two deltas sit at bits 7 and 23) & 0x07800780
//
// The subtraction never borrows across fields because delta <= emax.  Weights
// whose exact delta exceeds 15 (an exponent more than 15 binades below the
// largest of its group) decode to emax - 15 here and are corrected from the
// patch records; at 4 bits over 32 columns they are rare.
//
// Patch records: rows are grouped in tiles of 16; for every (tile, chunk)
// there is one record of 16-byte-aligned words at precs + ptile_off[tile *
// nchunks + chunk]:
//   words 0..31  emax of the 16 rows x 8 groups: byte 8 * row + group
//                (0 for rows past the end of the weight)
//   word 32      n_low (bits 0..15): entries in columns 0..127 of the chunk,
//                n_all (bits 16..31): all entries
//   word 33      n_q0 (bits 0..15): entries in columns 0..63,
//                n_q012 (bits 16..31): entries in columns 0..191
//   words 34..   entries grouped by 64-column quarter (quarter order; within
//                a quarter by row, then column), u32 each:
//                frag (bits 0..10) | half (bit 11) | exact bf16 bits << 16
//                where half = column >= 128 and frag is the element's 16-bit
//                slot in the mma fragment order of its half chunk (see
//                frag_index).
//   zero padding to a multiple of 4 words.
// ptile_off has n_tiles * nchunks + 1 entries; the last one is the total.
//
// Staged in shared memory, a chunk row is copied by TMA as three 128-byte
// lines with the 128-byte swizzle (16-byte unit u of line L lands at unit
// u ^ (L & 7) of its line, from a 1024-byte-aligned base): the 384-byte row
// pitch is a multiple of the 128-byte bank period, and without the swizzle
// lanes reading the same columns of different rows would share banks.
#pragma once

#include "bf16x_common.cuh"

namespace bf16x {

constexpr int kChunkElems = 256;
constexpr int kChunkBytes = 384;
constexpr int kChunkLines = kChunkBytes / 128;   // 128-byte lines per chunk row
constexpr int kSmOff = 0;
constexpr int kDOff = 256;
constexpr int kTileRows = 16;
constexpr int kRecHdr = 32;          // word index of the two header words
constexpr int kRecHdrWords = 34;     // words before the first entry
constexpr uint32_t kDeltaSat = 15u;

__host__ __device__ inline int64_t rec_words(int64_t n_entries) {
    return (kRecHdrWords + n_entries + 3) / 4 * 4;
}

__host__ __device__ inline int64_t resident_row_bytes(int64_t in_f) {
    return (in_f + kChunkElems - 1) / kChunkElems * kChunkBytes;
}

// Delta field of pair P of a group (4 words), positioned at bits 7..10 / 23..26.
template <int P>
__device__ __forceinline__ uint32_t pair_delta(const uint32_t (&dw)[4]) {
    return shl_signed<7 - 4 * (P & 3)>(dw[P >> 2]) & 0x07800780u;
}

// bf16x2 bits of pair P of a group: sm = the group's 8 sign|mant words,
// e2 = emax * 0x00800080 of the group.
template <int P>
__device__ __forceinline__ uint32_t decode_pair(const uint32_t (&sm)[8], const uint32_t (&dw)[4], uint32_t e2) {
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
                                                  const uint32_t (&dw)[4], uint32_t e2) {
    g.w[P] = decode_pair<P>(sm, dw, e2);
    if constexpr (P + 1 < 16) decode_pairs_from<P + 1>(g, sm, dw, e2);
}

__device__ __forceinline__ uint32_t emax_x2(uint32_t emax) { return emax * 0x00800080u; }

// Load group q of a chunk in its plain (unswizzled) form: global memory.
__device__ __forceinline__ void load_group(const uint8_t *chunk, int q, uint32_t (&sm)[8], uint32_t (&dw)[4]) {
    const uint4 a = *reinterpret_cast<const uint4 *>(chunk + kSmOff + 32 * q);
    const uint4 b = *reinterpret_cast<const uint4 *>(chunk + kSmOff + 32 * q + 16);
    const uint4 d = *reinterpret_cast<const uint4 *>(chunk + kDOff + 16 * q);
    sm[0] = a.x; sm[1] = a.y; sm[2] = a.z; sm[3] = a.w;
    sm[4] = b.x; sm[5] = b.y; sm[6] = b.z; sm[7] = b.w;
    dw[0] = d.x; dw[1] = d.y; dw[2] = d.z; dw[3] = d.w;
}

// Byte offsets, from the 1024-byte-aligned base of chunk rows staged with the
// 128-byte swizzle, of group q of row r: its two sign|mant units and its
// delta unit.
struct GroupOffsets {
    uint32_t a, b, d;
};

__host__ __device__ inline GroupOffsets sw_group_offsets(uint32_t r, uint32_t q) {
    const uint32_t la = kChunkLines * r + (q >> 2), ld = kChunkLines * r + 2u;
    GroupOffsets o;
    o.a = la * 128u + (((2u * (q & 3u)) ^ (la & 7u)) << 4);
    o.b = la * 128u + (((2u * (q & 3u) + 1u) ^ (la & 7u)) << 4);
    o.d = ld * 128u + ((q ^ (ld & 7u)) << 4);
    return o;
}

// Load group q of a row staged with the 128-byte swizzle (shared memory).
__device__ __forceinline__ void load_group_sw(const uint8_t *base, const GroupOffsets &o, uint32_t (&sm)[8],
                                              uint32_t (&dw)[4]) {
    const uint4 a = *reinterpret_cast<const uint4 *>(base + o.a);
    const uint4 b = *reinterpret_cast<const uint4 *>(base + o.b);
    const uint4 d = *reinterpret_cast<const uint4 *>(base + o.d);
    sm[0] = a.x; sm[1] = a.y; sm[2] = a.z; sm[3] = a.w;
    sm[4] = b.x; sm[5] = b.y; sm[6] = b.z; sm[7] = b.w;
    dw[0] = d.x; dw[1] = d.y; dw[2] = d.z; dw[3] = d.w;
}

// emax of group q of row r (0..15) from its record.
__device__ __forceinline__ uint32_t rec_emax(const uint32_t *rec, int r, int q) {
    return reinterpret_cast<const uint8_t *>(rec)[8 * r + q];
}

// Position of element (row, col) of a 16-row x 256-column chunk among the
// mma.m16n8k16 A fragments of its half (128 columns): 8 steps x 32 lanes x 4
// registers x 2 halves of 16 bits, as an 11-bit index.  Lane (g, t) holds
// rows g and g+8 of the 32-column group t; step J carries group columns
// 4J..4J+3 as pairs 2J (registers 0/1: rows g/g+8) and 2J+1 (registers 2/3).
// The index is (J * 32 + (lane ^ J)) * 8 + register * 2 + halfword; the
// patch entries carry it, and frag_position recovers (row, col) from it.
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

}  // namespace bf16x
