"""CPU oracle for the BF16X hot path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes wrapper over ``bf16x_oracle.c``, a plain-C restatement of
the reference algorithms (dfytensor/bfloat16x):

* ``quantize``      -> ``bf16x_quantize``            opqk_linear.py:291-324
* ``decode``        -> ``BF16XLinear._decode_tile``  opqk_linear.py:360-377
* ``decode_scatter``-> ``bf16x_decode_triton``       bf16x_triton_test.py:11-108
* ``linear``        -> ``BF16XLinear.forward``       opqk_linear.py:390-404
* ``gguf_*``        -> ``bf16x_gguf_block``          bf16x_gguf_block.py:44-187

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module; the product package never does.
Parity is pinned by ``tests/golden`` (vectors produced by the reference's own
Python code, see ``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libbf16x_oracle.so")
_lib = None


def build() -> str:
    """Compile the oracle with the committed Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or (
            os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_HERE, "bf16x_oracle.c"))
        ):
            build()
        _lib = ctypes.CDLL(_SO)
        i64, p = ctypes.c_int64, ctypes.c_void_p
        _lib.oracle_stream_words.restype = i64
        _lib.oracle_stream_words.argtypes = [i64, ctypes.c_int]
        _lib.oracle_quantize_sizes.argtypes = [p, i64, ctypes.c_int, p]
        _lib.oracle_quantize.argtypes = [p, i64, ctypes.c_int, p, p, p, p, p, p]
        _lib.oracle_decode.argtypes = [p, i64, p, i64, p, i64, p, p, p, i64,
                                       ctypes.c_int, i64, i64, p]
        _lib.oracle_matmul_bf16w.argtypes = [p, i64, p, i64, i64, p, p]
        _lib.oracle_linear.argtypes = [p, i64, p, i64, p, i64, p, p, p, i64,
                                       i64, i64, i64, p, i64, p, p]
        _lib.oracle_num_threads.restype = ctypes.c_int
        _lib.oracle_set_num_threads.argtypes = [ctypes.c_int]
        _lib.oracle_f32_to_bf16_bits.argtypes = [p, i64, p]
        _lib.oracle_gguf_quantize_blocks.argtypes = [p, i64, p]
        _lib.oracle_gguf_dequantize_blocks.argtypes = [p, i64, p]
        _lib.oracle_gguf_pack_ovf.restype = i64
        _lib.oracle_gguf_pack_ovf.argtypes = [p, i64, i64, p, p, p]
        _lib.oracle_gguf_apply_ovf.argtypes = [p, i64, i64, p, p, p]
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None and a.size else None


def stream_words(n: int, b: int) -> int:
    return int(lib().oracle_stream_words(n, b))


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


# --------------------------------------------------------------------------- #
# flat-stream BF16X                                                           #
# --------------------------------------------------------------------------- #
def quantize(bits: np.ndarray, out_f: int, in_f: int, sub: int = 16) -> dict:
    """bf16 bit patterns (uint16, out_f*in_f) -> the bf16x_quantize dict as numpy."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16).reshape(-1)
    n = bits.size
    assert n == out_f * in_f
    sizes = np.zeros(5, dtype=np.int64)
    lib().oracle_quantize_sizes(_ptr(bits), n, sub, _ptr(sizes))
    emax = np.zeros(int(sizes[0]), np.uint8)
    sign = np.zeros(int(sizes[1]), np.uint32)
    mant = np.zeros(int(sizes[2]), np.uint32)
    delta = np.zeros(int(sizes[3]), np.uint32)
    oi = np.zeros(int(sizes[4]), np.int32)
    ov = np.zeros(int(sizes[4]), np.uint8)
    if n:
        lib().oracle_quantize(_ptr(bits), n, sub, _ptr(emax), _ptr(sign), _ptr(mant),
                              _ptr(delta), _ptr(oi), _ptr(ov))
    return dict(emax=emax, sign_packed=sign.view(np.int32), mant_packed=mant.view(np.int32),
                delta_packed=delta.view(np.int32), delta_ovf_idx=oi, delta_ovf_val=ov,
                out_f=out_f, in_f=in_f, sub=sub)


def decode(p: dict, row_start: int = 0, row_end: int | None = None, sub: int = 16) -> np.ndarray:
    """Decode rows [row_start, row_end) of a dict -> uint16 bf16 bits [rows, in_f]."""
    out_f, in_f = int(p["out_f"]), int(p["in_f"])
    if row_end is None:
        row_end = out_f
    s = np.ascontiguousarray(np.asarray(p["sign_packed"]).view(np.uint32))
    m = np.ascontiguousarray(np.asarray(p["mant_packed"]).view(np.uint32))
    d = np.ascontiguousarray(np.asarray(p["delta_packed"]).view(np.uint32))
    e = np.ascontiguousarray(np.asarray(p["emax"]), dtype=np.uint8)
    oi = np.ascontiguousarray(np.asarray(p["delta_ovf_idx"]), dtype=np.int32)
    ov = np.ascontiguousarray(np.asarray(p["delta_ovf_val"]), dtype=np.uint8)
    cnt = (row_end - row_start) * in_f
    out = np.zeros(cnt, np.uint16)
    if cnt:
        lib().oracle_decode(_ptr(s), s.size, _ptr(m), m.size, _ptr(d), d.size, _ptr(e),
                            _ptr(oi), _ptr(ov), oi.size, sub, row_start * in_f, cnt, _ptr(out))
    return out.reshape(row_end - row_start, in_f)


def decode_scatter(p: dict, sub: int = 16) -> np.ndarray:
    """The reference's two-kernel decode (bf16x_triton_test.py:11-108):
    every element decodes with its stream delta (7 = saturated), then each
    overflow entry rewrites the exponent of the element at its own index,
    exp = clamp(emax - val, 0, 255) (_bf16x_fix_ovf_kernel, :55-77).  Unlike
    ``decode`` (searchsorted), it is exact for a table reduced to the
    entries with delta > 7, as the on-disk format stores it
    (pack_to_disk.py:62-66).  Returns uint16 bits [out_f, in_f]."""
    q = dict(p)
    q["delta_ovf_idx"] = np.zeros(0, np.int32)
    q["delta_ovf_val"] = np.zeros(0, np.uint8)
    out = decode(q, sub=sub).reshape(-1)
    oi = np.asarray(p["delta_ovf_idx"]).astype(np.int64)
    ov = np.asarray(p["delta_ovf_val"]).astype(np.int64)
    if oi.size:
        e = np.asarray(p["emax"]).astype(np.int64)[oi // sub]
        ex = np.clip(e - ov, 0, 255).astype(np.uint16)
        cur = out[oi]
        out[oi] = (cur & np.uint16(0x807F)) | (ex << np.uint16(7))
    return out.reshape(int(p["out_f"]), int(p["in_f"]))


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def matmul_bf16w(x: np.ndarray, w_bits: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """y = x @ W.T with W as bf16 bits [out, in], x fp32 [M, in]; fp32 result."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    M, in_f = x.shape
    out_f = w_bits.shape[0]
    y = np.zeros((M, out_f), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().oracle_matmul_bf16w(_ptr(x), M, _ptr(w_bits), out_f, in_f, _ptr(b), _ptr(y))
    return y


def linear(p: dict, x: np.ndarray, bias: np.ndarray | None = None, tile: int = 1024) -> np.ndarray:
    """Tile-wise decode + matmul (the reference CPU forward path)."""
    out_f, in_f = int(p["out_f"]), int(p["in_f"])
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, in_f)
    s = np.ascontiguousarray(np.asarray(p["sign_packed"]).view(np.uint32))
    m = np.ascontiguousarray(np.asarray(p["mant_packed"]).view(np.uint32))
    d = np.ascontiguousarray(np.asarray(p["delta_packed"]).view(np.uint32))
    e = np.ascontiguousarray(np.asarray(p["emax"]), dtype=np.uint8)
    oi = np.ascontiguousarray(np.asarray(p["delta_ovf_idx"]), dtype=np.int32)
    ov = np.ascontiguousarray(np.asarray(p["delta_ovf_val"]), dtype=np.uint8)
    y = np.zeros((x.shape[0], out_f), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().oracle_linear(_ptr(s), s.size, _ptr(m), m.size, _ptr(d), d.size, _ptr(e), _ptr(oi),
                        _ptr(ov), oi.size, out_f, in_f, tile, _ptr(x), x.shape[0], _ptr(b), _ptr(y))
    return y


# --------------------------------------------------------------------------- #
# GGUF block format                                                           #
# --------------------------------------------------------------------------- #
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.shape, np.uint16)
    lib().oracle_f32_to_bf16_bits(_ptr(x), x.size, _ptr(out))
    return out


def gguf_quantize_blocks(x: np.ndarray) -> np.ndarray:
    """fp32 (..., 32k) -> uint8 blocks (..., k, 46)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.shape[-1] % 32 == 0
    out = np.zeros(x.size // 32 * 46, np.uint8)
    lib().oracle_gguf_quantize_blocks(_ptr(x), x.size, _ptr(out))
    return out.reshape(*x.shape[:-1], x.shape[-1] // 32, 46)


def gguf_dequantize_bits(blocks: np.ndarray) -> np.ndarray:
    """uint8 blocks (..., k, 46) -> bf16 bits (..., 32k)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = b.size // 46
    out = np.zeros(nb * 32, np.uint16)
    lib().oracle_gguf_dequantize_blocks(_ptr(b), nb, _ptr(out))
    return out.reshape(*b.shape[:-2], b.shape[-2] * 32)


def gguf_dequantize_blocks(blocks: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(gguf_dequantize_bits(blocks))


def gguf_pack_ovf_arrays(bits: np.ndarray):
    """bf16 bits (rows, cols) -> (row_off u32[rows+1], cols u16[n], bits u16[n])."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    rows, cols = bits.shape
    n = int(lib().oracle_gguf_pack_ovf(_ptr(bits), rows, cols, None, None, None))
    ro = np.zeros(rows + 1, np.uint32)
    ec = np.zeros(n, np.uint16)
    eb = np.zeros(n, np.uint16)
    lib().oracle_gguf_pack_ovf(_ptr(bits), rows, cols, _ptr(ro), _ptr(ec), _ptr(eb))
    return ro, ec, eb


def gguf_pack_ovf(x: np.ndarray, bf16_exact: bool = False) -> bytes:
    """Serialised side table: u32 rows, u32 n, u32 row_off[rows+1], {u16 col, u16 bits}[n]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if bf16_exact:
        bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    else:
        bits = f32_to_bf16_bits(x)
    ro, ec, eb = gguf_pack_ovf_arrays(bits)
    ent = np.stack([ec, eb], axis=1).astype(np.uint16) if ec.size else np.zeros((0, 2), np.uint16)
    hdr = np.array([bits.shape[0], ec.size], np.uint32)
    return hdr.tobytes() + ro.tobytes() + ent.tobytes()


def gguf_apply_ovf_bits(decoded_bits: np.ndarray, blob: bytes) -> np.ndarray:
    hdr = np.frombuffer(blob[:8], np.uint32)
    rows, n = int(hdr[0]), int(hdr[1])
    ro = np.frombuffer(blob[8:8 + 4 * (rows + 1)], np.uint32).copy()
    ent = np.frombuffer(blob[8 + 4 * (rows + 1):8 + 4 * (rows + 1) + 4 * n], np.uint16).reshape(-1, 2)
    out = np.ascontiguousarray(decoded_bits, dtype=np.uint16).copy()
    cols = out.shape[1]
    ec = np.ascontiguousarray(ent[:, 0])
    eb = np.ascontiguousarray(ent[:, 1])
    lib().oracle_gguf_apply_ovf(_ptr(out), rows, cols, _ptr(ro), _ptr(ec), _ptr(eb))
    return out
