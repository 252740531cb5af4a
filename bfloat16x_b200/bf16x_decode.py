"""Standalone decode, drop-in for ``bf16x_decode_triton``
(bf16x_triton_test.py:80-108).

Same arguments and result (a [out_f, in_f] bf16 tensor on the GPU, bit-exact),
but the base decode and the overflow fix are one CUDA kernel
(``bf16x_decode`` of the C ABI): no host-side filtering of the table, no
``.item()`` synchronisation, no second launch.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import call, ptr


def bf16x_decode_triton(sign, mant, delta, emax, out_f, in_f, ovf_idx=None, ovf_val=None, sub=16,
                        out: torch.Tensor | None = None):
    """Decode flat BF16X streams into bf16 [out_f, in_f] on the streams' GPU."""
    if int(sub) != 16:
        raise ValueError("only sub=16 is supported (the reference kernel hard-codes 16)")
    dev = sign.device if sign.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if not torch.cuda.is_available():
        raise _lib.Bf16xError("bf16x_decode_triton needs a CUDA device")

    def dv(t, dt):
        return t.to(device=dev, dtype=dt, non_blocking=True).contiguous()

    s, m, d = dv(sign, torch.int32), dv(mant, torch.int32), dv(delta, torch.int32)
    e = dv(emax, torch.uint8)
    if ovf_idx is not None and ovf_val is not None and ovf_idx.numel() > 0:
        oi, ov = dv(ovf_idx, torch.int32), dv(ovf_val, torch.uint8)
        n_ovf = oi.numel()
    else:
        oi = ov = None
        n_ovf = 0
    if out is None:
        out = torch.empty((int(out_f), int(in_f)), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        call("bf16x_decode", ptr(s), s.numel(), ptr(m), m.numel(), ptr(d), d.numel(), ptr(e), e.numel(),
             ptr(oi), ptr(ov), n_ovf, int(out_f), int(in_f), 16, ptr(out),
             torch.cuda.current_stream(dev).cuda_stream)
    return out


bf16x_decode = bf16x_decode_triton

__all__ = ["bf16x_decode_triton", "bf16x_decode"]
