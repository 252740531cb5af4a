"""BF16X packer and the decode+matmul Linear, drop-in for the BF16X half of the
reference's ``opqk_linear`` module.

* ``bf16x_quantize`` (opqk_linear.py:291-324) -- same dict, same dtypes, same
  stream lengths, bit for bit; packed on the GPU by ``bf16x_quantize_count`` /
  ``bf16x_quantize`` of the C ABI.  Returned on the CPU like the reference
  (``device=`` keeps it elsewhere).
* ``BF16XLinear`` (opqk_linear.py:327-407) -- same constructors
  (``BF16XLinear(linear)`` / ``BF16XLinear.from_packed(b, ...)``) and the same
  ``decode_to_bf16`` / ``clear_bf16`` / ``decoded_weight`` methods, but the
  forward runs the fused CUDA kernels on the resident layout instead of the
  reference's per-tile torch decode + matmul.
* ``replace_with_bf16x`` (opqk_linear.py:428-440) -- same walk; failures are
  raised instead of being silently skipped.

The OPQ-K lossy quantizer of the reference module is a different format and
is not part of this package.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from ._lib import call, ptr, require_cuda, stream_of

SUB = 16
_KEYS = ("emax", "sign_packed", "mant_packed", "delta_packed", "delta_ovf_idx", "delta_ovf_val")


def stream_words(n: int, bits: int) -> int:
    """Words of a pack_bits_stream stream of n values (opqk_linear.py:53-64)."""
    return int(_lib.lib().bf16x_stream_words(int(n), int(bits)))


@torch.no_grad()
def bf16x_quantize(w: torch.Tensor, sub: int = SUB, device=None) -> dict:
    """bf16 weight [out_f, in_f] -> BF16X dict (see opqk_linear.py:291-324).

    The packing runs on the GPU (the weight's device if it is a CUDA tensor,
    else the current CUDA device).  The dict is returned on ``device``
    (default: CPU, as the reference does)."""
    if sub != SUB:
        raise ValueError("only sub=16 is supported (the reference decoders hard-code 16)")
    if w.dim() != 2:
        raise ValueError("bf16x_quantize expects a 2-D weight [out_f, in_f]")
    out_f, in_f = w.shape
    if not torch.cuda.is_available():
        raise _lib.Bf16xError("bf16x_quantize packs on the GPU; no CUDA device is available")
    dev = w.device if w.is_cuda else torch.device("cuda", torch.cuda.current_device())
    wb = w.detach().to(device=dev, dtype=torch.bfloat16).contiguous().reshape(-1)
    n = wb.numel()
    L = _lib.lib()
    n_sign, n_mant, n_delta = (int(L.bf16x_stream_words(n, b)) for b in (1, 7, 3))
    n_emax = (n + sub - 1) // sub
    st = torch.cuda.current_stream(dev).cuda_stream
    scratch = torch.empty(int(L.bf16x_quantize_scratch_bytes(n)) // 8 + 1, dtype=torch.int64, device=dev)
    total = torch.zeros(1, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        call("bf16x_quantize_count", ptr(wb), n, sub, ptr(scratch), ptr(total), st)
        n_ovf = int(total.item())
        emax = torch.empty(n_emax, dtype=torch.uint8, device=dev)
        sign = torch.empty(n_sign, dtype=torch.int32, device=dev)
        mant = torch.empty(n_mant, dtype=torch.int32, device=dev)
        delta = torch.empty(n_delta, dtype=torch.int32, device=dev)
        oi = torch.empty(n_ovf, dtype=torch.int32, device=dev)
        ov = torch.empty(n_ovf, dtype=torch.uint8, device=dev)
        call("bf16x_quantize", ptr(wb), n, sub, ptr(scratch), ptr(emax), ptr(sign), ptr(mant), ptr(delta),
             ptr(oi) if n_ovf else None, ptr(ov) if n_ovf else None, n_ovf, st)
    target = torch.device("cpu") if device is None else torch.device(device)
    out = dict(emax=emax, sign_packed=sign, mant_packed=mant, delta_packed=delta,
               delta_ovf_idx=oi, delta_ovf_val=ov)
    out = {k: v.to(target).contiguous() for k, v in out.items()}
    out.update(out_f=int(out_f), in_f=int(in_f), sub=sub)
    return out


def packed_nbytes(p: dict) -> int:
    """Bytes of a dict as the reference accounts them (5 bytes per overflow entry,
    bf16x_fused.py:254-256)."""
    return (p["sign_packed"].numel() * 4 + p["mant_packed"].numel() * 4 + p["delta_packed"].numel() * 4
            + p["emax"].numel() + p["delta_ovf_idx"].numel() * 5)


class BF16XLinear(nn.Module):
    """Decode+matmul Linear on a BF16X dict (opqk_linear.py:327-407), GPU-only.

    ``forward`` runs the fused decode+GEMV (<= 16 rows of activations) or
    decode+GEMM kernel on the resident layout; ``decode_to_bf16`` caches the
    exact bf16 weight, after which ``forward`` is a plain ``F.linear`` as in
    the reference."""

    def __init__(self, orig_linear: nn.Linear, sub: int = SUB, tile: int = 1024):
        super().__init__()
        b = bf16x_quantize(orig_linear.weight.data, sub=sub)
        bias = orig_linear.bias.data if orig_linear.bias is not None else None
        self._init_from_buffers(b, sub, tile, bias)

    @classmethod
    def from_packed(cls, b: dict, sub: int = SUB, tile: int = 1024, bias=None, alphas=None):
        obj = cls.__new__(cls)
        nn.Module.__init__(obj)
        obj._init_from_buffers(b, sub, tile, bias)
        return obj

    def _init_from_buffers(self, b, sub, tile, bias):
        from .resident import ResidentWeight
        self.out_f, self.in_f = int(b["out_f"]), int(b["in_f"])
        self.sub, self.tile = sub, tile
        self._w_bf16 = None
        self.resident = ResidentWeight.from_packed(b)
        if bias is not None:
            self.bias = nn.Parameter(bias.detach().clone().to(self.resident.device), requires_grad=False)
        else:
            self.register_parameter("bias", None)

    @property
    def weight(self):
        return torch.zeros(1, 1, dtype=torch.bfloat16, device=self.resident.device)

    def _decode_tile(self, s, e):
        """Exact bf16 rows [s, e) of the weight, [e - s, in_f] on the device
        (opqk_linear.py:360-377 decodes the same rows from the flat streams)."""
        return self.resident.decode_rows(s, e)

    def decode_to_bf16(self):
        self._w_bf16 = self.resident.decode()
        return self._w_bf16

    def clear_bf16(self):
        self._w_bf16 = None

    def decoded_weight(self):
        return self.resident.decode().to(torch.float32)

    def forward(self, x):
        if self._w_bf16 is not None:
            return torch.nn.functional.linear(x, self._w_bf16, self.bias)
        return self.resident.linear(x, self.bias)


def replace_with_bf16x(module: nn.Module, sub: int = SUB, tile: int = 1024, count=None, min_el: int = 50000) -> int:
    """Replace every nn.Linear with more than ``min_el`` weights (opqk_linear.py:428-440)."""
    if count is None:
        count = [0]
    for name, child in list(module.named_children()):
        if isinstance(child, nn.Linear) and child.weight.numel() > min_el:
            setattr(module, name, BF16XLinear(child, sub=sub, tile=tile))
            count[0] += 1
        else:
            replace_with_bf16x(child, sub, tile, count, min_el)
    return count[0]


def _check_dict(p: dict) -> None:
    missing = [k for k in _KEYS + ("out_f", "in_f") if k not in p]
    if missing:
        raise KeyError(f"BF16X dict is missing {missing}")


__all__ = ["bf16x_quantize", "BF16XLinear", "replace_with_bf16x", "stream_words", "packed_nbytes", "SUB"]
