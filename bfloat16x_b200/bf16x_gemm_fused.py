"""Drop-in for the reference's ``bf16x_gemm_fused`` module (bf16x_gemm_fused.py).

* ``bf16x_fused_gemm`` -- same arguments as the reference's multi-token
  fused decode+GEMM (bf16x_gemm_fused.py:97-114).  Like the reference, when
  no overflow table is passed the weights decode with saturated deltas
  (a stored 7 means emax - 7); pass ``ovf_idx`` / ``ovf_val`` (the dict's
  table) for the exact weights.  The activations are multiplied in bf16 on
  the tcgen05 tensor cores and the result is returned in x's dtype.  The
  resident layout is built on the first call for a set of stream tensors and
  cached by their addresses.  ``bn``, ``bk``, ``num_warps`` and
  ``num_stages`` are Triton tuning knobs of the reference kernel, accepted
  and ignored.
* ``Bf16xGemmLinear`` -- the prefill Linear (bf16x_gemm_fused.py:154-196):
  ``resident=True`` keeps the weight in HBM; ``resident=False`` keeps it in
  pinned host memory and copies it to a per-device staging buffer on every
  forward (stream-ordered, so the staging buffer is shared by all layers).
  Unlike the reference module the exact weights are used (patches applied).
* ``deploy_bf16x_gemm`` -- replaces the model's nn.Linear layers
  (bf16x_gemm_fused.py:199-242), same arguments and return value.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from .bf16x_fused import _linear_targets, _resident_from_streams, _set_module, cached_resident
from .resident import ResidentWeight

_CHUNK_MB = 1024


class _Pinner:
    """Pinned host storage handed out from chunks of ``_CHUNK_MB`` MiB, so
    that packing many layers makes few pinned allocations."""

    def __init__(self, chunk_mb: int = _CHUNK_MB):
        self.chunk = int(chunk_mb) << 20
        self.buf = None
        self.used = 0
        self.total = 0

    def add(self, t: torch.Tensor) -> torch.Tensor:
        t = t.detach().contiguous()
        n = t.numel() * t.element_size()
        off = (self.used + 255) // 256 * 256 if self.buf is not None else 0
        if self.buf is None or off + n > self.buf.numel():
            size = max(n, self.chunk)
            self.buf = torch.empty(size, dtype=torch.uint8, pin_memory=True)
            self.total += size
            off = 0
        v = self.buf[off:off + n].view(t.dtype).view(t.shape)
        v.copy_(t)
        self.used = off + n
        return v


_PIN = _Pinner()


def bf16x_fused_gemm(x, sign, mant, delta, emax, out_f, in_f, group=16,
                     bn=128, bk=32, num_warps=8, num_stages=1, ovf_idx=None, ovf_val=None):
    """y[M, out_f] = x[M, in_f] @ W^T with W decoded on the fly
    (bf16x_gemm_fused.py:97-114); y has x's dtype."""
    _lib.require_cuda(x, "x")
    if group != 16:
        raise ValueError("only 16-element sub-blocks are supported")
    M = x.numel() // int(in_f)
    dev = x.device
    has_ovf = ovf_idx is not None and ovf_idx.numel() > 0

    def build():
        if has_ovf:
            oi = ovf_idx.to(dev, torch.int32)
            ov = ovf_val.to(dev, torch.uint8)
        else:
            oi = torch.empty(0, dtype=torch.int32, device=dev)
            ov = torch.empty(0, dtype=torch.uint8, device=dev)
        return _resident_from_streams(sign.to(dev), mant.to(dev), delta.to(dev), emax.to(dev), oi, ov, out_f, in_f)

    streams = (sign, mant, delta, emax) + ((ovf_idx, ovf_val) if has_ovf else ())
    rw = cached_resident(("gemm", dev.index, int(out_f), int(in_f), has_ovf), streams, build)
    od = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
    y = rw.gemm(x.reshape(M, int(in_f)), out_dtype=od)
    return y.to(x.dtype)


# ------------------------------------------------------------------ #
#  staging of non-resident weights: one buffer per (device, stream)
# ------------------------------------------------------------------ #
_STAGING: dict = {}


def _staging(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _STAGING.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _STAGING[key] = buf
    return buf


class Bf16xGemmLinear(nn.Module):
    """BF16X prefill Linear (bf16x_gemm_fused.py:154-196).

    resident=True : the weight lives in HBM in the resident layout.
    resident=False: the resident layout lives in pinned host memory and is
                    copied to a shared device staging buffer on each forward;
                    the same kernels then consume it."""

    def __init__(self, packed: dict, bias: torch.Tensor | None = None, resident: bool = True, pin=None):
        super().__init__()
        if not torch.cuda.is_available():
            raise _lib.Bf16xError("Bf16xGemmLinear runs on a CUDA device (bfloat16x_b200 has no CPU path)")
        self.out_features = int(packed["out_f"])
        self.in_features = int(packed["in_f"])
        self.resident = bool(resident)
        dev = torch.device("cuda", torch.cuda.current_device())
        rw = ResidentWeight.from_packed(packed, device=dev)
        if bias is not None:
            self.register_buffer("_bias", bias.detach().clone().to(dev))
        else:
            self._bias = None
        if self.resident:
            self._gpu = rw
            self._cpu = None
        else:
            p = pin if pin is not None else _PIN
            self._gpu = None
            self._cpu = {"layout": p.add(rw.layout.cpu()), "ptile_off": p.add(rw.ptile_off.cpu()),
                         "precs": p.add(rw.precs.cpu())}
            self._shadow = None          # ResidentWeight over the staging buffer
            self._shadow_buf = None
            del rw

    def _stream_in(self, device: torch.device) -> ResidentWeight:
        c = self._cpu
        sizes = [c[k].numel() * c[k].element_size() for k in ("layout", "ptile_off", "precs")]
        offs = [0, (sizes[0] + 255) // 256 * 256]
        offs.append(offs[1] + (sizes[1] + 255) // 256 * 256)
        buf = _staging(device, offs[2] + sizes[2])
        if self._shadow is None or self._shadow_buf is not buf:
            lay = buf[offs[0]:offs[0] + sizes[0]].view(c["layout"].shape)
            pto = buf[offs[1]:offs[1] + sizes[1]].view(torch.int32)
            prc = buf[offs[2]:offs[2] + sizes[2]].view(torch.int32)
            self._shadow = ResidentWeight(lay, pto, prc, self.out_features, self.in_features)
            self._shadow_buf = buf
        s = self._shadow
        s.layout.copy_(c["layout"], non_blocking=True)
        s.ptile_off.copy_(c["ptile_off"], non_blocking=True)
        s.precs.copy_(c["precs"], non_blocking=True)
        return s

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            x = x.cuda()
        rw = self._gpu if self.resident else self._stream_in(x.device)
        od = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
        return rw.linear(x, self._bias, out_dtype=od).to(x.dtype)


@torch.no_grad()
def deploy_bf16x_gemm(model: nn.Module, min_numel: int = 1000, skip=("lm_head", "embed"),
                      resident_fn=None, verbose: bool = True):
    """Replace nn.Linear layers by Bf16xGemmLinear (bf16x_gemm_fused.py:199-242).
    ``resident_fn(name) -> bool`` picks HBM-resident or pinned-host streaming
    per layer (default: resident).  Returns (packed bytes, weights)."""
    from .opqk_linear import bf16x_quantize
    targets = _linear_targets(model, min_numel, skip)
    total = n_el = 0
    for name, mod in targets:
        w = mod.weight.data
        p = bf16x_quantize(w.to(torch.bfloat16), sub=16)
        bias = mod.bias.data if mod.bias is not None else None
        res = resident_fn(name) if resident_fn else True
        _set_module(model, name, Bf16xGemmLinear(p, bias=bias, resident=res))
        total += sum(p[k].numel() * p[k].element_size() for k in ("sign_packed", "mant_packed", "delta_packed", "emax"))
        total += p["delta_ovf_idx"].numel() * 5
        n_el += w.numel()
        mod.weight.data = torch.empty(0)
        del w, p
    if verbose:
        print(f"[bf16x-gemm] {len(targets)} layers | {total/1e6:.0f}MB packed "
              f"({n_el*2/max(total, 1):.2f}x vs bf16) | bpw={total*8/max(n_el, 1):.2f}", flush=True)
    return total, n_el


__all__ = ["bf16x_fused_gemm", "Bf16xGemmLinear", "deploy_bf16x_gemm"]
