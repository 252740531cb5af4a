"""ctypes binding of libbf16x_b200.so (the C ABI declared in include/bf16x_b200.h).

The CUDA library is the only compute path of this package: if it is missing,
every entry point raises.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# BF16X_LIB points at another build of the same library (e.g. a tuned variant)
LIB_PATH = os.environ.get("BF16X_LIB") or os.path.join(_HERE, "libbf16x_b200.so")

BF16X_DTYPE_BF16 = 0
BF16X_DTYPE_F32 = 1
BF16X_DTYPE_F32_TRUNC = 2
CHUNK_ELEMS = 256
CHUNK_BYTES = 384
TILE_ROWS = 16
REC_HDR_WORD = 32       # record word holding n_low | n_all << 16 (after 128 bytes of emax)
REC_ENTRY_WORD = 34     # first patch entry of a record


class Bf16xError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


_i64, _i32, _p, _u32p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)

# name -> (restype, argtypes)
_SIGS = {
    "bf16x_version": (_i32, []),
    "bf16x_last_error": (ctypes.c_char_p, []),
    "bf16x_device_status": (_i32, [_i32, _u32p]),
    "bf16x_decode": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i32, _p, _p]),
    "bf16x_stream_words": (_i64, [_i64, _i32]),
    "bf16x_quantize_scratch_bytes": (_i64, [_i64]),
    "bf16x_quantize_count": (_i32, [_p, _i64, _i32, _p, _p, _p]),
    "bf16x_quantize": (_i32, [_p, _i64, _i32, _p, _p, _p, _p, _p, _p, _p, _i64, _p]),
    "bf16x_resident_row_bytes": (_i64, [_i64]),
    "bf16x_repack_count": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                  _p, _p]),
    "bf16x_repack": (_i32, [_p, _i64, _p, _i64, _p, _i64, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64,
                            _p, _p, _p, _p]),
    "bf16x_resident_decode": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _p]),
    "bf16x_gemv_scratch_bytes": (_i64, [_i64, _i64]),
    "bf16x_gemv": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _i32, _i64, _p, _p, _i64, _p]),
    "bf16x_gemv_noalloc_max_rows": (_i64, []),
    "bf16x_gemv_noalloc": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _i32, _i64, _p]),
    "bf16x_gguf_quantize": (_i32, [_p, _i32, _i64, _p, _p]),
    "bf16x_gguf_dequantize": (_i32, [_p, _i64, _p, _i32, _p]),
    "bf16x_gguf_ovf_count": (_i32, [_p, _i32, _i64, _i64, _p, _p]),
    "bf16x_gguf_ovf_pack": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _p]),
    "bf16x_gguf_apply_ovf": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _i64, _p]),
    "bf16x_gguf_side_index_count": (_i32, [_p, _p, _i64, _i64, _i64, _p, _p]),
    "bf16x_gguf_side_index": (_i32, [_p, _p, _p, _i64, _i64, _i64, _p, _p, _p]),
    "bf16x_gguf_gemv_scratch_bytes": (_i64, [_i64, _i64]),
    "bf16x_gguf_gemv": (_i32, [_p, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _i32, _i64, _p, _p, _i64, _p]),
    "bf16x_gemm": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _i32, _i64, _p]),
    "bf16x_gemm_workspace_bytes": (_i64, [_i64, _i64, _i64]),
    "bf16x_gemm_ws": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _i32, _i64, _p, _i64, _p]),
    "bf16x_selftest_wait": (_i32, [_i32, _i64, _p, _p, _p]),
    "bf16x_gemv_peers": (_i32, [_p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _i32, _p, _i64, _i64, _i64, _i32, _i32,
                                _p, _i32, _i64, _p, _p, _p, _i64, _p]),
    "bf16x_add_rmsnorm": (_i32, [_p, _p, _p, ctypes.c_float, _i64, _i64, _p, _p, _p]),
    "bf16x_rope_qkv": (_i32, [_p, _i64, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p, _i64, _i64, _p]),
    "bf16x_silu_mul": (_i32, [_p, _i64, _i64, _p, _p]),
    "bf16x_peer_handle_bytes": (_i64, []),
    "bf16x_peer_export": (_i32, [_p, _p, _p]),
    "bf16x_peer_import": (_i32, [_p, _p]),
    "bf16x_peer_close": (_i32, [_p]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load the CUDA library, failing loudly when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise Bf16xError(
                f"{LIB_PATH} is missing: build it with `python -m bfloat16x_b200.build` "
                "(nvcc, sm_100a). bfloat16x_b200 has no CPU fallback.")
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(l, name)
            fn.restype = res
            fn.argtypes = args
        _lib = l
    return _lib


def exported_symbols() -> list:
    return list(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().bf16x_last_error().decode(errors="replace")
        raise Bf16xError(f"{what} failed ({rc}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def device_status(device: int | None = None) -> int:
    """Read and clear device-side error bits (synchronises the device)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    flags = ctypes.c_uint32(0)
    check(lib().bf16x_device_status(dev, ctypes.byref(flags)), "bf16x_device_status")
    return int(flags.value)


def check_device_status(device: int | None = None) -> None:
    f = device_status(device)
    if f:
        from .resident import reset_workspaces
        reset_workspaces()
        names = {1: "wait timeout", 2: "overflow index not ascending", 4: "overflow index out of range",
                 8: "bad resident layout", 16: "device-side index out of range"}
        what = ", ".join(v for k, v in names.items() if f & k) or hex(f)
        raise Bf16xError(f"device reported: {what} (flags {f:#x})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise Bf16xError(f"{name} must be a CUDA tensor (bfloat16x_b200 runs on the GPU only)")
