"""Drop-in for the reference's ``bf16x_gguf_block`` (the llama.cpp
GGML_TYPE_BF16X block format and its lossless side table), computed on the
GPU through the C ABI.

Same names and semantics as bf16x_gguf_block.py: numpy arrays in give numpy
arrays out (the work runs on the current CUDA device); CUDA tensors in give
CUDA tensors out with no host copies.  ``GgufWeight`` adds what the reference
leaves to llama.cpp: a device-resident GGUF weight that feeds the fused
decode+GEMV / decode+GEMM kernels (the 11.5-bpw GGUF-block variant of the
matmul path), exact when the side table is given.

Block (46 bytes per 32 weights): emax[2] (per 16-weight half, floored at 7),
sign[4], mant[28], delta[12], all LSB-first; delta 7 is the zero marker.
Side table blob: u32 n_rows, u32 n_entries, u32 row_off[n_rows + 1],
{u16 col, u16 bf16_bits}[n_entries] sorted by row then column.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import BF16X_DTYPE_BF16, BF16X_DTYPE_F32, BF16X_DTYPE_F32_TRUNC, call, ptr

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
    the GPU kernels; ``resident()`` re-encodes those exact values once into
    the kernel layout so the fused decode+GEMV / decode+GEMM kernels consume
    the GGUF variant (its zero-marked and side-table weights become patches)."""

    def __init__(self, blocks: torch.Tensor, out_f: int, in_f: int, side=None):
        if in_f % QK_BF16X:
            raise ValueError(f"in_f {in_f} not divisible by {QK_BF16X}")
        self.blocks = blocks.contiguous()
        self.out_f, self.in_f = int(out_f), int(in_f)
        self.side = side                       # (row_off, cols, bits) device tensors or None
        self._resident = None

    @classmethod
    @torch.no_grad()
    def from_float(cls, w, lossless: bool = True) -> "GgufWeight":
        t, mode = _values_on_device(w)
        out_f, in_f = t.shape
        blocks = torch.empty(out_f * in_f // QK_BF16X * BLOCK_BYTES, dtype=torch.uint8, device=t.device)
        with torch.cuda.device(t.device):
            call("bf16x_gguf_quantize", ptr(t), mode, t.numel(), ptr(blocks), _stream(t.device))
        side = _pack_ovf_dev(t, mode, out_f, in_f) if lossless else None
        return cls(blocks, out_f, in_f, side)

    @classmethod
    def from_blocks(cls, blocks, out_f: int, in_f: int, blob: bytes | None = None) -> "GgufWeight":
        dev = _device()
        b = torch.from_numpy(np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)).to(dev) \
            if not isinstance(blocks, torch.Tensor) else blocks.reshape(-1).to(dev)
        side = None
        if blob is not None:
            rows, ro, ec, eb = _blob_to_device(blob, dev)
            if rows != out_f:
                raise ValueError(f"side table has {rows} rows, weight {out_f}")
            side = (ro, ec, eb)
        return cls(b, out_f, in_f, side)

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

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None, out_dtype=None) -> torch.Tensor:
        return self.resident().linear(x, bias, out_dtype)


__all__ = ["QK_BF16X", "BLOCK_BYTES", "OVF_HDR_BYTES", "fp32_to_bf16_bits", "bf16_bits_to_fp32",
           "quantize_blocks", "dequantize_blocks", "quantize_tensor", "pack_ovf", "pack_ovf_tensors",
           "unpack_ovf", "apply_ovf", "dequantize_lossless", "ovf_overflow_mask", "ovf_stats", "GgufWeight"]
