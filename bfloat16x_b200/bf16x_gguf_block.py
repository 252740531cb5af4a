"""Drop-in for the reference's ``bf16x_gguf_block`` (the llama.cpp
GGML_TYPE_BF16X block format and its lossless side table), computed on the
GPU through the C ABI.

Same names and semantics as bf16x_gguf_block.py: numpy arrays in give numpy
arrays out (the work runs on the current CUDA device); CUDA tensors in give
CUDA tensors out with no host copies.  ``GgufWeight`` adds what the reference
leaves to llama.cpp: a device-resident GGUF weight whose GEMV reads the
46-byte blocks in place (the 11.5-bpw GGUF-block variant of the matmul
path, exact when the side table is given) and whose larger batches run on
the tensor-core GEMM.

Block (46 bytes per 32 weights): emax[2] (per 16-weight half, floored at 7),
sign[4], mant[28], delta[12], all LSB-first; delta 7 is the zero marker.
Side table blob: u32 n_rows, u32 n_entries, u32 row_off[n_rows + 1],
{u16 col, u16 bf16_bits}[n_entries] sorted by row then column.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import (BF16X_DTYPE_BF16, BF16X_DTYPE_F32, BF16X_DTYPE_F32_TRUNC, Bf16xError, call, check_device_status,
                   lib, ptr)

QK_BF16X = 32
BLOCK_BYTES = 46
OVF_HDR_BYTES = 8


# ------------------------------------------------------------------ helpers
def fp32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, nearest-even with quiet NaNs (host helper,
    bf16x_gguf_block.py:45-50)."""
    n = np.asarray(x, dtype=np.float32).view(np.uint32)
    n = np.where((n & 0x7FFFFFFF) > 0x7F800000, (n & np.uint32(0xFFFF0000)) | np.uint32(64 << 16), n)
    return ((n.astype(np.uint64) + (0x7FFF + ((n >> 16) & 1))) >> 16).astype(np.uint16)


def bf16_bits_to_fp32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> exact float32 (host helper)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise _lib.Bf16xError("bfloat16x_b200 runs on a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _values_on_device(x, bf16_exact: bool = False):
    """(device tensor, x_dtype code) for float data given as numpy or torch."""
    if isinstance(x, torch.Tensor):
        t = x.detach()
        dev = t.device if t.is_cuda else _device()
        if t.dtype == torch.bfloat16:
            return t.to(dev).contiguous(), BF16X_DTYPE_BF16
        t = t.to(device=dev, dtype=torch.float32).contiguous()
    else:
        dev = _device()
        t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(dev)
    return t, (BF16X_DTYPE_F32_TRUNC if bf16_exact else BF16X_DTYPE_F32)


def _bits_u16(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int16)


# ---------------------------------------------------------------- blocks
def quantize_blocks(x):
    """float array (..., 32k) -> uint8 blocks (..., k, 46) (bf16x_gguf_block.py:64-81)."""
    is_np = not isinstance(x, torch.Tensor)
    t, mode = _values_on_device(x)
    shape = tuple(t.shape)
    if shape[-1] % QK_BF16X:
        raise ValueError(f"last dim {shape[-1]} not divisible by {QK_BF16X}")
    n = t.numel()
    out = torch.empty((n // QK_BF16X) * BLOCK_BYTES, dtype=torch.uint8, device=t.device)
    with torch.cuda.device(t.device):
        call("bf16x_gguf_quantize", ptr(t), mode, n, ptr(out), _stream(t.device))
    out = out.view(*shape[:-1], shape[-1] // QK_BF16X, BLOCK_BYTES)
    return out.cpu().numpy() if is_np else out


def _dequantize_dev(b: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    nb = b.numel() // BLOCK_BYTES
    ydt = BF16X_DTYPE_F32 if out_dtype == torch.float32 else BF16X_DTYPE_BF16
    y = torch.empty(nb * QK_BF16X, dtype=out_dtype, device=b.device)
    with torch.cuda.device(b.device):
        call("bf16x_gguf_dequantize", ptr(b), nb, ptr(y), ydt, _stream(b.device))
    return y


def dequantize_blocks(packed, out_dtype: torch.dtype = torch.float32):
    """uint8 blocks (..., k, 46) -> values (..., 32k) (bf16x_gguf_block.py:84-95);
    float32 like the reference, or bf16 for CUDA tensors with out_dtype."""
    is_np = not isinstance(packed, torch.Tensor)
    b = torch.from_numpy(np.ascontiguousarray(packed, dtype=np.uint8)).to(_device()) if is_np \
        else packed.to(_device() if not packed.is_cuda else packed.device).contiguous()
    if b.shape[-1] != BLOCK_BYTES:
        raise ValueError(f"blocks must end in a dimension of {BLOCK_BYTES} bytes")
    y = _dequantize_dev(b, torch.float32 if is_np else out_dtype)
    y = y.view(*b.shape[:-2], b.shape[-2] * QK_BF16X)
    return y.cpu().numpy() if is_np else y


def quantize_tensor(x):
    """Quantize a full weight whose last dimension is a multiple of 32."""
    cols = x.shape[-1]
    if cols % QK_BF16X:
        raise ValueError(f"last dim {cols} not divisible by {QK_BF16X}")
    return quantize_blocks(x)


# ------------------------------------------------------------ side table
def _pack_ovf_dev(t: torch.Tensor, mode: int, rows: int, cols: int):
    """(row_off uint32 [rows+1], cols uint16 [n], bits uint16 [n]) on the device."""
    dev = t.device
    row_off = torch.empty(rows + 1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = _stream(dev)
        call("bf16x_gguf_ovf_count", ptr(t), mode, rows, cols, ptr(row_off), st)
        n = int(row_off[rows].item())
        ec = torch.empty(max(n, 1), dtype=torch.int16, device=dev)
        eb = torch.empty(max(n, 1), dtype=torch.int16, device=dev)
        if n:
            call("bf16x_gguf_ovf_pack", ptr(t), mode, rows, cols, ptr(row_off), ptr(ec), ptr(eb), st)
    return row_off, ec[:n], eb[:n]


def pack_ovf_tensors(x, bf16_exact: bool = False):
    """Side table of a (rows, cols) weight as device tensors
    (row_off int32 [rows+1], cols int16 [n], bits int16 [n])."""
    t, mode = _values_on_device(x, bf16_exact)
    if t.dim() != 2:
        raise ValueError("pack_ovf expects a (rows, cols) weight")
    rows, cols = t.shape
    if cols % QK_BF16X:
        raise ValueError(f"cols {cols} not divisible by {QK_BF16X}")
    return _pack_ovf_dev(t, mode, rows, cols)


def _serialize(rows: int, row_off: torch.Tensor, ec: torch.Tensor, eb: torch.Tensor) -> bytes:
    ro = row_off.cpu().numpy().astype(np.uint32)
    n = int(ro[-1]) if ro.size else 0
    ent = np.empty((n, 2), dtype=np.uint16)
    if n:
        ent[:, 0] = ec.cpu().numpy().view(np.uint16)
        ent[:, 1] = eb.cpu().numpy().view(np.uint16)
    hdr = np.array([rows, n], dtype=np.uint32)
    return hdr.tobytes() + ro.tobytes() + ent.tobytes()


def pack_ovf(x, bf16_exact: bool = False) -> bytes:
    """(rows, cols) weight -> serialized side table (bf16x_gguf_block.py:143-161)."""
    row_off, ec, eb = pack_ovf_tensors(x, bf16_exact)
    return _serialize(row_off.numel() - 1, row_off, ec, eb)


def unpack_ovf(blob: bytes):
    """-> (n_rows, row_off, cols, bf16 bits) (bf16x_gguf_block.py:164-171); host parse."""
    hdr = np.frombuffer(blob[:OVF_HDR_BYTES], dtype=np.uint32)
    rows, n = int(hdr[0]), int(hdr[1])
    off = OVF_HDR_BYTES
    row_off = np.frombuffer(blob[off:off + 4 * (rows + 1)], dtype=np.uint32)
    off += 4 * (rows + 1)
    ent = np.frombuffer(blob[off:off + 4 * n], dtype=np.uint16).reshape(-1, 2)
    return rows, row_off, ent[:, 0], ent[:, 1]


def _blob_to_device(blob: bytes, dev):
    rows, row_off, cols, bits = unpack_ovf(blob)
    ro = torch.from_numpy(row_off.astype(np.int32)).to(dev)
    ec = torch.from_numpy(np.ascontiguousarray(cols).view(np.int16).copy()).to(dev)
    eb = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).to(dev)
    return rows, ro, ec, eb


def _apply_dev(y: torch.Tensor, rows: int, cols: int, ro, ec, eb) -> None:
    ydt = BF16X_DTYPE_F32 if y.dtype == torch.float32 else BF16X_DTYPE_BF16
    with torch.cuda.device(y.device):
        call("bf16x_gguf_apply_ovf", ptr(y), ydt, rows, cols, ptr(ro), ptr(ec), ptr(eb), ec.numel(),
             _stream(y.device))


def apply_ovf(decoded, blob: bytes):
    """Copy of a dequantized (rows, cols) tensor with the side table's exact
    values written back (bf16x_gguf_block.py:174-181)."""
    is_np = not isinstance(decoded, torch.Tensor)
    dev = _device() if is_np or not decoded.is_cuda else decoded.device
    y = (torch.from_numpy(np.ascontiguousarray(decoded, dtype=np.float32)) if is_np else decoded).to(dev).clone()
    rows, ro, ec, eb = _blob_to_device(blob, dev)
    if y.shape[0] != rows:
        raise ValueError(f"side table has {rows} rows, tensor {tuple(y.shape)}")
    _apply_dev(y, rows, y.shape[1], ro, ec, eb)
    return y.cpu().numpy() if is_np else y


def dequantize_lossless(packed, blob: bytes):
    """Blocks + side table -> exact float32 weights, flattened
    (bf16x_gguf_block.py:184-188)."""
    rows = int(unpack_ovf(blob)[0])
    dec = dequantize_blocks(packed)
    n = dec.size if isinstance(dec, np.ndarray) else dec.numel()
    return apply_ovf(dec.reshape(rows, n // max(rows, 1)), blob).reshape(-1)


def ovf_overflow_mask(x, bf16_exact: bool = False) -> np.ndarray:
    """(rows, cols) bool mask of the elements quantize_blocks clamps."""
    t, mode = _values_on_device(x, bf16_exact)
    rows, cols = t.shape
    row_off, ec, _ = _pack_ovf_dev(t, mode, rows, cols)
    mask = torch.zeros((rows, cols), dtype=torch.bool, device=t.device)
    counts = (row_off[1:] - row_off[:-1]).to(torch.int64)
    r = torch.repeat_interleave(torch.arange(rows, device=t.device), counts)
    mask[r, ec.to(torch.int64) & 0xFFFF] = True
    return mask.cpu().numpy()


def ovf_stats(x):
    """-> (n_overflow, n_elements)."""
    t, mode = _values_on_device(x)
    row_off, _, _ = _pack_ovf_dev(t, mode, t.shape[0], t.shape[1])
    return int(row_off[-1].item()), t.numel()


# ------------------------------------------------- device-resident weight
class GgufWeight:
    """A (out_f, in_f) weight in GGUF BF16X blocks on the device, with an
    optional lossless side table.  ``dequantize()`` gives bf16 bits through
    the GPU kernels.  ``gemv()`` multiplies 1..16 rows of activations either
    by the blocks in place (``bf16x_gguf_gemv``: 11.5 bits per weight
    streamed, the side table's exact values stored over the decoded weights;
    in_f a multiple of 256) or through ``resident()``, the exact values
    re-encoded once into the kernel layout (its zero-marked and side-table
    weights become patches), which the tensor-core GEMM always uses.

    ``native=None`` picks the faster GEMV for the weight: the blocks in place
    without a side table (the lossy 11.5-bpw format), the resident layout with
    one (a table's entries, a few percent of the weights, cost the in-place
    kernel more than the resident layout's few patches); True or False forces
    either."""

    def __init__(self, blocks: torch.Tensor, out_f: int, in_f: int, side=None, native: bool | None = None):
        if in_f % QK_BF16X:
            raise ValueError(f"in_f {in_f} not divisible by {QK_BF16X}")
        self.blocks = blocks.contiguous()
        self.out_f, self.in_f = int(out_f), int(in_f)
        self.side = side                       # (row_off, cols, bits) device tensors or None
        self.native = native
        self._resident = None
        self._items = None                     # side table as per-item records (block GEMV)
        self._tile_counters = None
        self._scratch_need = None
        self._stream_bytes = None

    @classmethod
    @torch.no_grad()
    def from_float(cls, w, lossless: bool = True, native: bool | None = None) -> "GgufWeight":
        t, mode = _values_on_device(w)
        out_f, in_f = t.shape
        blocks = torch.empty(out_f * in_f // QK_BF16X * BLOCK_BYTES, dtype=torch.uint8, device=t.device)
        with torch.cuda.device(t.device):
            call("bf16x_gguf_quantize", ptr(t), mode, t.numel(), ptr(blocks), _stream(t.device))
        side = _pack_ovf_dev(t, mode, out_f, in_f) if lossless else None
        return cls(blocks, out_f, in_f, side, native=native)

    @classmethod
    def from_blocks(cls, blocks, out_f: int, in_f: int, blob: bytes | None = None,
                    native: bool | None = None) -> "GgufWeight":
        dev = _device()
        b = torch.from_numpy(np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)).to(dev) \
            if not isinstance(blocks, torch.Tensor) else blocks.reshape(-1).to(dev)
        side = None
        if blob is not None:
            rows, ro, ec, eb = _blob_to_device(blob, dev)
            if rows != out_f:
                raise ValueError(f"side table has {rows} rows, weight {out_f}")
            side = (ro, ec, eb)
        return cls(b, out_f, in_f, side, native=native)

    @property
    def device(self) -> torch.device:
        return self.blocks.device

    def nbytes(self) -> int:
        n = self.blocks.numel()
        if self.side is not None:
            n += OVF_HDR_BYTES + 4 * self.side[0].numel() + 4 * self.side[1].numel()
        return n

    def bits_per_weight(self) -> float:
        return 8.0 * self.nbytes() / max(1, self.out_f * self.in_f)

    def dequantize(self) -> torch.Tensor:
        """bf16 weight [out_f, in_f]: lossy (zero marker) without a side table,
        exact with one."""
        y = _dequantize_dev(self.blocks, torch.bfloat16).view(self.out_f, self.in_f)
        if self.side is not None:
            ro, ec, eb = self.side
            _apply_dev(y, self.out_f, self.in_f, ro, ec, eb)
        return y

    def resident(self):
        """The weight in the fused kernels' resident layout (built once)."""
        if self._resident is None:
            from .opqk_linear import bf16x_quantize
            from .resident import ResidentWeight
            w = self.dequantize()
            p = bf16x_quantize(w, device=self.device)
            self._resident = ResidentWeight.from_packed(p, device=self.device)
        return self._resident

    @property
    def blocks_native(self) -> bool:
        """True when the block GEMV can read this weight in place (in_f % 256 == 0)."""
        return self.in_f % 256 == 0 and self.in_f <= 65536

    @property
    def gemv_in_place(self) -> bool:
        """True when gemv() runs on the blocks in place (see ``native``)."""
        if not self.blocks_native:
            return False
        if self.native is not None:
            return bool(self.native)
        return self.side is None or self.side[1].numel() == 0

    def _stream(self) -> int:
        return _stream(self.device)

    @torch.no_grad()
    def side_records(self):
        """(item_off, item_recs): the side table re-indexed into one record per
        (16-row tile, 256-column chunk) for the block GEMV, built once on the
        GPU; (None, None) without a table or entries."""
        if self._items is None:
            if self.side is None or self.side[1].numel() == 0:
                self._items = (None, None)
            else:
                ro, ec, eb = self.side
                dev = self.device
                T = (self.out_f + 15) // 16 * (self.in_f // 256)
                item_off = torch.empty(T + 1, dtype=torch.int32, device=dev)
                with torch.cuda.device(dev):
                    call("bf16x_gguf_side_index_count", ptr(ro), ptr(ec), self.out_f, self.in_f, ec.numel(),
                         ptr(item_off), self._stream())
                    check_device_status(dev.index)
                    words = int(item_off[-1].item())
                    recs = torch.empty(max(words, 4), dtype=torch.int32, device=dev)
                    call("bf16x_gguf_side_index", ptr(ro), ptr(ec), ptr(eb), self.out_f, self.in_f, ec.numel(),
                         ptr(item_off), ptr(recs), self._stream())
                self._items = (item_off, recs)
        return self._items

    def gemv(self, x: torch.Tensor, bias: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[b, n] = sum_k W[n, k] x[b, k] (+ bias) for 1..16 rows of
        activations, decoded from the blocks in place (side table applied)."""
        from .resident import GEMV_MAX_BATCH, gemv_scratch
        if not self.gemv_in_place:
            return self.resident().gemv(x, bias, out_dtype=out_dtype, out=out)
        if not x.is_cuda:
            raise Bf16xError("x must be a CUDA tensor (bfloat16x_b200 runs on the GPU only)")
        x2 = x.reshape(-1, self.in_f).to(torch.bfloat16)
        B = x2.shape[0]
        if B < 1 or B > GEMV_MAX_BATCH:
            raise ValueError(f"gemv takes 1..{GEMV_MAX_BATCH} rows of activations, got {B}")
        if not (x2.is_contiguous() and x2.data_ptr() % 16 == 0):
            x2 = x2.contiguous().clone()
        if out is None:
            out = torch.empty((B, self.out_f), dtype=out_dtype, device=self.device)
        ydt = BF16X_DTYPE_F32 if out.dtype == torch.float32 else BF16X_DTYPE_BF16
        b = None if bias is None else bias.to(device=self.device, dtype=torch.bfloat16).contiguous()
        item_off, recs = self.side_records()
        with torch.cuda.device(self.device):
            if self._tile_counters is None:
                self._tile_counters = torch.zeros((self.out_f + 15) // 16 + 1, dtype=torch.int32, device=self.device)
                self._scratch_need = int(lib().bf16x_gguf_gemv_scratch_bytes(self.out_f, self.in_f))
            ws = gemv_scratch(self.device, self._scratch_need)
            call("bf16x_gguf_gemv", ptr(self.blocks), self.out_f, self.in_f, ptr(item_off), ptr(recs), ptr(x2), B,
                 x2.stride(0), ptr(b), ptr(out), ydt, out.stride(0), ptr(self._tile_counters), ptr(ws), ws.numel(),
                 self._stream())
        return out

    def stream_bytes(self) -> int:
        """Bytes one gemv() reads for the weight: in place, the blocks plus the
        side-table records and their offsets when there are entries; else the
        resident layout's."""
        if not self.gemv_in_place:
            return self.resident().nbytes()
        if self._stream_bytes is None:
            n = self.blocks.numel()
            item_off, recs = self.side_records()
            if recs is not None:
                n += 4 * item_off.numel() + 4 * int(item_off[-1].item())
            self._stream_bytes = n
        return self._stream_bytes

    def gemm(self, x: torch.Tensor, bias: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        """Any number of rows on the tensor-core GEMM (resident layout)."""
        return self.resident().gemm(x, bias, out_dtype=out_dtype, out=out)

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None, out_dtype=None) -> torch.Tensor:
        """x[..., in_f] -> [..., out_f]: the block GEMV for up to 16 rows of
        activations, the resident tensor-core GEMM above that."""
        from .resident import GEMV_MAX_BATCH
        x2 = x.reshape(-1, self.in_f)
        if x2.shape[0] <= GEMV_MAX_BATCH and self.gemv_in_place:
            od = out_dtype or (x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16)
            return self.gemv(x2, bias, out_dtype=od).reshape(*x.shape[:-1], self.out_f)
        return self.resident().linear(x, bias, out_dtype)


__all__ = ["QK_BF16X", "BLOCK_BYTES", "OVF_HDR_BYTES", "fp32_to_bf16_bits", "bf16_bits_to_fp32",
           "quantize_blocks", "dequantize_blocks", "quantize_tensor", "pack_ovf", "pack_ovf_tensors",
           "unpack_ovf", "apply_ovf", "dequantize_lossless", "ovf_overflow_mask", "ovf_stats", "GgufWeight"]
