/*
 * bf16x_b200.h -- C ABI of the B200-native BF16X hot path.
 *
 * Plain pointers and sizes, no framework types.  All pointers are device
 * pointers unless stated otherwise; `stream` is a cudaStream_t.  Every
 * function returns BF16X_OK (0) or a negative status; bf16x_last_error()
 * returns the message of the last failure on the calling host thread.
 * Nothing allocates device memory except where a function says so.
 *
 * The reference (dfytensor/bfloat16x) has no C ABI: its boundary is a Python
 * API.  Each entry point below names the reference function it replaces
 * (file:line within the reference project); the Python package
 * bfloat16x_b200 mirrors those Python functions on top of this ABI.
 *
 * Formats
 *   flat streams   : the bf16x_quantize dict (opqk_linear.py:291-324): LSB-first
 *                    int32 bit streams sign (1 b/elt), mant (7 b), delta (3 b,
 *                    7 = saturated), emax (u8 per 16 flat elements), overflow
 *                    table idx (int32 ascending flat positions) + val (u8 true
 *                    delta, >= 7).
 *   resident layout: the kernel layout built once per weight by bf16x_repack:
 *                    rows of ceil(in_f/256) chunks of 384 bytes
 *                    ([256 B sign|mant bytes][128 B pair-aligned 4-bit deltas]),
 *                    12 bits per weight, plus one record per (16-row tile,
 *                    256-column chunk): the emax of each 32-column group of
 *                    its rows (128 B), two header words of per-quarter entry
 *                    counts, then u32 entries for the weights whose exact
 *                    exponent delta exceeds 15,
 *                    mma-fragment slot (11 b) | column half << 11 | exact bf16 << 16,
 *                    sorted by (64-column quarter, row, column).
 *   GGUF blocks    : 46-byte blocks of 32 weights (bf16x_gguf_block.py:6-17).
 */
#ifndef BF16X_B200_H
#define BF16X_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BF16X_OK               0
#define BF16X_ERR_INVALID     -1   /* bad argument (size, alignment, dtype) */
#define BF16X_ERR_CUDA        -2   /* CUDA runtime error */
#define BF16X_ERR_UNSUPPORTED -3   /* shape or device not supported */
#define BF16X_ERR_DEVICE      -4   /* a kernel reported a device-side error */

#define BF16X_DTYPE_BF16 0
#define BF16X_DTYPE_F32  1
/* float32 input whose values are bf16-exact: the high half is taken as is
 * (the reference's bf16_exact=True, bf16x_gguf_block.py:115-120) */
#define BF16X_DTYPE_F32_TRUNC 2

#define BF16X_CHUNK_ELEMS 256
#define BF16X_CHUNK_BYTES 384

/* ---- library ----------------------------------------------------------- */
int bf16x_version(void);
const char *bf16x_last_error(void);

/* Read and clear the device-side status bits that kernels of this library
 * set on `device` (wait timeouts, malformed overflow tables).  Synchronises
 * the device.  *flags == 0 means no error was recorded. */
int bf16x_device_status(int device, uint32_t *flags);

/* ---- flat-stream decode ------------------------------------------------ */
/* Replaces bf16x_decode_triton (bf16x_triton_test.py:80-108): base decode and
 * overflow fix in ONE kernel.  out: bf16 bits [out_f * in_f].  Stream word
 * counts may be the exact dict lengths or padded ones; nothing past them is
 * read.  ovf_idx/ovf_val are device arrays (n_ovf may be 0).  Semantics are
 * those of BF16XLinear._decode_tile (opqk_linear.py:360-377) for well-formed
 * tables: exponent = (emax - d) & 0xFF with d the true delta of listed
 * elements.  sub must be 16. */
int bf16x_decode(const uint32_t *sign, int64_t n_sign_words,
                 const uint32_t *mant, int64_t n_mant_words,
                 const uint32_t *delta, int64_t n_delta_words,
                 const uint8_t *emax, int64_t n_emax,
                 const int32_t *ovf_idx, const uint8_t *ovf_val, int64_t n_ovf,
                 int64_t out_f, int64_t in_f, int sub,
                 uint16_t *out, void *stream);

/* ---- GPU packer --------------------------------------------------------- */
/* Replaces bf16x_quantize (opqk_linear.py:291-324) on the device.  Two calls:
 * bf16x_quantize_count writes the number of overflow entries (delta >= 7) to
 * *n_ovf_dev (device int64) using `scratch` (bf16x_quantize_scratch_bytes(n)
 * bytes, device); bf16x_quantize then fills the streams, whose lengths follow
 * the reference's pack_bits_stream rule (opqk_linear.py:53-64), and the
 * overflow table (capacity entries at most).  w: bf16 bits [n]. */
int64_t bf16x_stream_words(int64_t n, int bits);
int64_t bf16x_quantize_scratch_bytes(int64_t n);
int bf16x_quantize_count(const uint16_t *w, int64_t n, int sub, void *scratch,
                         int64_t *n_ovf_dev, void *stream);
int bf16x_quantize(const uint16_t *w, int64_t n, int sub, const void *scratch,
                   uint8_t *emax, uint32_t *sign, uint32_t *mant, uint32_t *delta,
                   int32_t *ovf_idx, uint8_t *ovf_val, int64_t capacity, void *stream);

/* ---- resident layout ---------------------------------------------------- */
/* Replaces the per-layer device preparation of Bf16xFused.__init__
 * (bf16x_fused.py:154-192: _pad1 + CSR build) and Bf16xGemmLinear.__init__
 * (bf16x_gemm_fused.py:163-184).  Rows [row0, row1) of the flat dict are
 * decoded exactly (overflow applied) and re-encoded into the resident layout:
 * row-major chunks of 384 bytes, and one record per (16-row tile, 256-column
 * chunk) holding the groups' emax and the weights whose exact exponent delta
 * exceeds 15.
 *   bf16x_resident_row_bytes: bytes per row of the layout.
 *   bf16x_repack_count: record sizes -> ptile_off[0..n_tiles*n_chunks]
 *                       (device int32, exclusive scan in words; the last
 *                       entry is the total record words).
 *   bf16x_repack: writes layout [rows][row_bytes] and the records (u32).
 * in_f must be <= 65536. */
int64_t bf16x_resident_row_bytes(int64_t in_f);
int bf16x_repack_count(const uint32_t *sign, int64_t n_sign_words,
                       const uint32_t *mant, int64_t n_mant_words,
                       const uint32_t *delta, int64_t n_delta_words,
                       const uint8_t *emax, int64_t n_emax,
                       const int32_t *ovf_idx, const uint8_t *ovf_val, int64_t n_ovf,
                       int64_t out_f, int64_t in_f, int64_t row0, int64_t row1,
                       int32_t *ptile_off, void *stream);
int bf16x_repack(const uint32_t *sign, int64_t n_sign_words,
                 const uint32_t *mant, int64_t n_mant_words,
                 const uint32_t *delta, int64_t n_delta_words,
                 const uint8_t *emax, int64_t n_emax,
                 const int32_t *ovf_idx, const uint8_t *ovf_val, int64_t n_ovf,
                 int64_t out_f, int64_t in_f, int64_t row0, int64_t row1,
                 const int32_t *ptile_off, uint8_t *layout, uint32_t *precs,
                 void *stream);

/* Resident layout -> bf16 bits [rows][ld_out] (bit-exact, patches applied).
 * Used by the two-segment path (Bf16xFused 'opt' mode, bf16x_fused.py:194-205). */
int bf16x_resident_decode(const uint8_t *layout, const int32_t *ptile_off,
                          const uint32_t *precs, int64_t rows, int64_t in_f,
                          uint16_t *out, int64_t ld_out, void *stream);

/* ---- fused decode + GEMV (batch 1..16) ---------------------------------- */
/* Replaces bf16x_fused_gemv / _bf16x_gemv_fused_kernel (bf16x_fused.py:32-127):
 * y[b][n] = sum_k W[n][k] * x[b][k] (+ bias[n]) for b < batch <= 16, with W
 * read from the resident layout and decoded in registers, patches applied
 * exactly, fp32 accumulation, deterministic.  x: bf16 [batch][ldx],
 * ldx >= ceil(in_f/256)*256 elements with zeros past in_f, rows 16-byte
 * aligned.  bias: bf16 [rows] or NULL.  y: [batch][ldy] of y_dtype.
 * tile_counters: ceil(rows/16) int32 owned by the weight, zero-filled once;
 * every successful call leaves them zero.  scratch: bf16x_gemv_scratch_bytes
 * (rows, in_f) bytes of device memory (for the current device) holding the
 * partial sums of tiles that several warps share; no initialisation needed.
 * Calls that may overlap on the GPU need their own counters and scratch. */
int64_t bf16x_gemv_scratch_bytes(int64_t rows, int64_t in_f);
int bf16x_gemv(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
               int64_t rows, int64_t in_f,
               const uint16_t *x, int64_t batch, int64_t ldx,
               const uint16_t *bias, void *y, int y_dtype, int64_t ldy,
               int32_t *tile_counters, void *scratch, int64_t scratch_bytes, void *stream);

/* No counterpart in the reference.  bf16x_gemv without caller-supplied
 * device memory, for callers that cannot allocate: a plain C host or FFI
 * binding with no device allocator of its own, or a serving loop that must
 * not call cudaMalloc/cudaFree (which synchronise the device) once running.
 * Same arguments and results as bf16x_gemv otherwise, but batch 1..8 only
 * (9..16 rows fail with BF16X_ERR_INVALID: their partial sums are twice as
 * large); nothing is allocated.  The tile counters and partial sums live in
 * one fixed device array of this library (2 MiB of partial sums + 128 KiB of
 * counters per device), so rows <= bf16x_gemv_noalloc_max_rows() (524288);
 * larger requests fail with BF16X_ERR_UNSUPPORTED.  Each call clears its counters on
 * `stream` before the launch.  The first call on a device looks up that
 * array's address (cudaGetSymbolAddress), so make it before any stream
 * capture.  All calls on a device share the one array: calls that can
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. */
int64_t bf16x_gemv_noalloc_max_rows(void);
int bf16x_gemv_noalloc(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                       int64_t rows, int64_t in_f,
                       const uint16_t *x, int64_t batch, int64_t ldx,
                       const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *stream);

/* ---- tensor parallel over NVLink: GEMV with the exchange inside -------- */
/* Tensor parallelism over the nranks GPUs of one node (2..8).  The reference
 * has no multi-GPU path; this replaces bf16x_fused_gemv
 * (bf16x_fused.py:114-127) followed by a separate all-gather or all-reduce.
 * bf16x_gemv_peers is bf16x_gemv whose epilogue sends every output, as one
 * 64-bit word (fp32 bits | launch epoch << 32, a single-copy-atomic store, so
 * no fence or flag is needed), to ll[q] of every rank q (ll: host array of
 * nranks device pointers, 8-byte aligned, ll[rank] on this GPU, the others
 * peer memory mapped with bf16x_peer_import):
 *   mode 0 (gather, row-sharded weight): this rank holds rows
 *     [row0, row0 + rows) of an out_total-row weight; words go to
 *     ll[q][b * ll_ld + row0 + row];
 *   mode 1 (reduce, column-sharded weight): rows == out_total, row0 == 0;
 *     this rank's partial sums go to ll[q][(rank * batch + b) * ll_ld + row].
 * Every GPU then waits (bounded) for the words of its own ll[rank] that carry
 * this launch's epoch and writes y [batch][ldy] (y_dtype, ldy >= out_total):
 * the gathered rows, or the sum of the partials in rank order.  The kernel
 * completes once y is whole.  The exchange buffers must start zeroed
 * (batch * ll_ld words, mode 1: nranks * batch * ll_ld); the launch epoch
 * lives in state (this GPU's two zeroed u32 words), shared by the collective
 * GEMVs of one group, which must run in the same order on every rank, on one
 * stream each; a buffer used by one launch must not be used by the next one.
 * Every rank needs rows >= 1.  bias applies to this rank's rows (give NULL in
 * mode 1 and add it once after). */
int bf16x_gemv_peers(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                     int64_t rows, int64_t in_f, const uint16_t *x, int64_t batch, int64_t ldx,
                     const uint16_t *bias, int mode, uint64_t *const *ll, int64_t ll_ld,
                     int64_t out_total, int64_t row0, int nranks, int rank, void *y, int y_dtype,
                     int64_t ldy, uint32_t *state, int32_t *tile_counters, void *scratch,
                     int64_t scratch_bytes, void *stream);

/* CUDA IPC plumbing for the peer pointers above (no counterpart in the
 * reference).  bf16x_peer_export: the IPC handle (bf16x_peer_handle_bytes()
 * bytes, host) of the device allocation holding ptr and ptr's offset in it.
 * bf16x_peer_import: maps another process's handle on the current device
 * (lazy peer access) and returns the allocation's base; a handle imported
 * twice shares one mapping.  bf16x_peer_close: releases one import. */
int64_t bf16x_peer_handle_bytes(void);
int bf16x_peer_export(const void *ptr, void *handle, int64_t *offset);
int bf16x_peer_import(const void *handle, void **base);
int bf16x_peer_close(void *base);

/* ---- fused decode + GEMM (tcgen05, prefill) ----------------------------- */
/* Replaces bf16x_fused_gemm / _bf16x_gemm_fused_kernel
 * (bf16x_gemm_fused.py:31-114): y[m][n] = sum_k x[m][k] * W[n][k] (+ bias[n])
 * for m < M tokens, W decoded tile by tile into shared memory (exact: the
 * patches are applied, unlike the reference's saturated decode) and
 * multiplied on the tensor cores (tcgen05.mma, fp32 accumulation in tensor
 * memory).  x: bf16 [M][ldx], ldx >= in_f and a multiple of 8, 16-byte
 * aligned; columns past in_f are never read.  bias: bf16 [rows] or NULL.
 * y: [M][ldy] of y_dtype. */
int bf16x_gemm(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
               int64_t rows, int64_t in_f,
               const uint16_t *x, int64_t M, int64_t ldx,
               const uint16_t *bias, void *y, int y_dtype, int64_t ldy, void *stream);

/* Workspace that lets bf16x_gemm_ws decode each 256-row slab of the weight
 * once for all token tiles (instead of once per tile): 0 when the shape does
 * not use it (fewer than 1024 tokens, or fewer tiles than CTA pairs). */
int64_t bf16x_gemm_workspace_bytes(int64_t rows, int64_t in_f, int64_t M);
/* bf16x_gemm with a device workspace of bf16x_gemm_workspace_bytes(rows,
 * in_f, M) bytes, 256-byte aligned, not shared with a call that may run at
 * the same time; its contents need no initialisation.  NULL: same as
 * bf16x_gemm. */
int bf16x_gemm_ws(const uint8_t *layout, const int32_t *ptile_off, const uint32_t *precs,
                  int64_t rows, int64_t in_f,
                  const uint16_t *x, int64_t M, int64_t ldx,
                  const uint16_t *bias, void *y, int y_dtype, int64_t ldy,
                  void *workspace, int64_t workspace_bytes, void *stream);

/* ---- GGUF BF16X block format (llama.cpp GGML_TYPE_BF16X) --------------- */
/* 32 weights per 46-byte block: emax[2] (per 16-weight half, floored at 7),
 * sign[4], mant[28], delta[12]; delta 7 is the zero marker.  x_dtype:
 * BF16X_DTYPE_BF16 (bf16 bits), BF16X_DTYPE_F32 (rounded to nearest even,
 * NaNs quieted, as bf16x_gguf_block.py:45-50) or BF16X_DTYPE_F32_TRUNC.
 * Replaces quantize_blocks (bf16x_gguf_block.py:64-81): n % 32 == 0,
 * blocks: n/32 x 46 bytes, 4-byte aligned. */
int bf16x_gguf_quantize(const void *x, int x_dtype, int64_t n, uint8_t *blocks, void *stream);
/* Replaces dequantize_blocks (bf16x_gguf_block.py:84-95): y gets
 * nblocks*32 values, bf16 bits or float32 (y_dtype). */
int bf16x_gguf_dequantize(const uint8_t *blocks, int64_t nblocks, void *y, int y_dtype, void *stream);
/* Lossless side table, replaces pack_ovf (bf16x_gguf_block.py:143-161) in two
 * steps.  bf16x_gguf_ovf_count writes row_off[0..rows] (rows+1 uint32): entry
 * offsets per row, row_off[rows] = number of entries (cols % 32 == 0, cols <=
 * 65536).  bf16x_gguf_ovf_pack then writes the entries: column (u16) and
 * exact bf16 bits (u16), sorted by row then column. */
int bf16x_gguf_ovf_count(const void *x, int x_dtype, int64_t rows, int64_t cols, uint32_t *row_off,
                         void *stream);
int bf16x_gguf_ovf_pack(const void *x, int x_dtype, int64_t rows, int64_t cols, const uint32_t *row_off,
                        uint16_t *ecols, uint16_t *ebits, void *stream);
/* Replaces apply_ovf (bf16x_gguf_block.py:174-181): writes each entry's
 * exact value into y [rows][cols] (bf16 bits or float32). */
int bf16x_gguf_apply_ovf(void *y, int y_dtype, int64_t rows, int64_t cols, const uint32_t *row_off,
                         const uint16_t *ecols, const uint16_t *ebits, int64_t n_entries, void *stream);

/* ---- GEMV on the GGUF blocks in place ------------------------------------ */
/* The decode+GEMV of llama.cpp's BF16X matmul with the lossless side table
 * applied (GGML_OP_SPARSE_MM, README.md:311-318; block decode
 * bf16x_gguf_block.py:84-95, table bf16x_gguf_block.py:107-181) reading the
 * 46-byte blocks themselves: y[b][n] = sum_k W[n][k] x[b][k] (+ bias[n]) for
 * batch 1..16, W the blocks (rows x in_f/32 blocks, row-major, 16-byte
 * aligned; in_f a multiple of 256, <= 65536) decoded exactly, with the side
 * table's values where it has entries.  The side table is first re-indexed
 * into one record per (16-row tile, 256-column chunk):
 * bf16x_gguf_side_index_count writes item_off[0..T] (T = ceil(rows/16) *
 * in_f/256, int32 word offsets, item_off[T] = words of records), then
 * bf16x_gguf_side_index fills item_recs (item_off[T] uint32, 16-byte
 * aligned) from the table (row_off: rows+1 u32; cols, bits: u16 per entry,
 * sorted by row then column).  A table with bad offsets, unsorted columns or
 * columns >= in_f is reported through the device status.  Without a table
 * (the lossy format) item_off and item_recs are both NULL.  x: [batch][ldx]
 * bf16 bits (ldx >= in_f, multiple of 8, 16-byte aligned); tile_counters:
 * ceil(rows/16) int32 zeroed once (the kernel leaves them zero); scratch:
 * bf16x_gguf_gemv_scratch_bytes(rows, in_f) bytes, 16-byte aligned. */
int bf16x_gguf_side_index_count(const uint32_t *row_off, const uint16_t *cols, int64_t rows, int64_t in_f,
                                int64_t n_entries, int32_t *item_off, void *stream);
int bf16x_gguf_side_index(const uint32_t *row_off, const uint16_t *cols, const uint16_t *bits, int64_t rows,
                          int64_t in_f, int64_t n_entries, const int32_t *item_off, uint32_t *item_recs,
                          void *stream);
int64_t bf16x_gguf_gemv_scratch_bytes(int64_t rows, int64_t in_f);
int bf16x_gguf_gemv(const uint8_t *blocks, int64_t rows, int64_t in_f, const int32_t *item_off,
                    const uint32_t *item_recs, const uint16_t *x, int64_t batch, int64_t ldx,
                    const uint16_t *bias, void *y, int y_dtype, int64_t ldy, int32_t *tile_counters,
                    void *scratch, int64_t scratch_bytes, void *stream);

/* ---- decoder glue --------------------------------------------------------- */
/* No counterpart in the reference (it has no decoder of its own).  The
 * element-wise steps between the projections of the end-to-end Llama-style
 * decoder that measures the hot path in a model, one kernel each instead of a
 * few dozen framework kernels per layer (bf16 in and out, fp32 arithmetic).
 * bf16x_add_rmsnorm: per row of n, h = x + delta (delta may be NULL: h = x,
 *   h_out unused), y = h * rsqrt(mean(h^2) + eps) * w.
 * bf16x_rope_qkv: qkv [tokens][(H + 2 KV) * D] of batch rows of T tokens at
 *   positions *pos0 .. *pos0 + T - 1 (device int64): q and k heads rotated
 *   pairwise (cos/sin tables fp32 [positions][D/2]), q to q_out [tokens][H][D],
 *   k and v to cache_k / cache_v at [b][position] (batch stride cache_ld_b
 *   elements, KV * D per position).  Positions must lie in [0, max_pos) (the
 *   cache's and the tables' length); a token outside is skipped and sets a
 *   status bit (bf16x_device_status).
 * bf16x_silu_mul: out [rows][F] = silu(gu[r][i]) * gu[r][F + i]. */
int bf16x_add_rmsnorm(const uint16_t *x, const uint16_t *delta, const uint16_t *w, float eps, int64_t rows,
                      int64_t n, uint16_t *h_out, uint16_t *y, void *stream);
int bf16x_rope_qkv(const uint16_t *qkv, int64_t tokens, int T, int H, int KV, int D, const int64_t *pos0,
                   const float *cos_t, const float *sin_t, uint16_t *q_out, uint16_t *cache_k,
                   uint16_t *cache_v, int64_t cache_ld_b, int64_t max_pos, void *stream);
int bf16x_silu_mul(const uint16_t *gu, int64_t rows, int64_t F, uint16_t *out, void *stream);

/* ---- self-test of the bounded waits ------------------------------------- */
/* No counterpart in the reference.  Runs one of the library's bounded device
 * waits -- which: 0 the GEMV's mbarrier wait, 1 the tcgen05 GEMM roles' wait,
 * 2 the slab GEMM's cross-CTA counter wait, 3 the collective GEMV's wait for
 * its exchange words -- against a fresh mbarrier that nothing completes (0, 1), until the
 * u32 *flag reaches 1 (2), or until the 64-bit word at flag (8-byte aligned)
 * carries epoch 1 in its high half (3), with a limit of limit_ns (1 us ..
 * 100 ms).
 * result (device int32[3]): gave up (1/0), abort flag raised (1/0),
 * microseconds waited.  A wait that gives up sets the wait-timeout bit read by
 * bf16x_device_status; the kernel returns and the context stays usable. */
int bf16x_selftest_wait(int which, int64_t limit_ns, const uint32_t *flag, int32_t *result, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BF16X_B200_H */
