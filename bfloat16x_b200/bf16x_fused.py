"""Drop-in for the reference's ``bf16x_fused`` module (bf16x_fused.py).

* ``bf16x_fused_gemv`` -- same arguments as the reference's single-token
  fused decode+GEMV (bf16x_fused.py:114-127): the flat streams plus the
  per-row CSR of overflow corrections (``olk`` column, ``old`` true delta,
  ``oloff`` row offsets).  It runs the sm_100a decode+GEMV kernel on the
  resident layout, which it builds from those tensors on the first call and
  caches for as long as the same tensor objects live unmodified (the
  reference modules build their CSR once at ``__init__`` the same way).  ``r``, ``bk``, ``group`` and ``num_warps`` are
  Triton tuning knobs of the reference kernel; they are accepted and ignored.
* ``Bf16xFused`` -- the three-mode Linear (bf16x_fused.py:149-229):
  ``'fused'`` runs the fused kernels (decode+GEMV for up to 16 rows of
  activations, the tcgen05 decode+GEMM above that; the reference falls back
  to decode + F.linear for more than one row), ``'opt'`` decodes into a
  process-wide shared buffer and calls F.linear, ``'repo'`` runs the
  stand-alone decode with the overflow table kept on the host and calls
  F.linear.
* ``deploy_bf16x_fused`` -- replaces the model's nn.Linear layers
  (bf16x_fused.py:232-263), with the same skip rule and return value.

Everything computes on the GPU through the C ABI; there is no CPU path.
"""
from __future__ import annotations

import weakref
from collections import OrderedDict

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .bf16x_decode import bf16x_decode_triton
from .resident import ResidentWeight

_CACHE_SLOTS = 256
# address key -> _CacheEntry.  An entry is used only while every stream tensor
# it was built from is the same live object at the same version: torch's
# caching allocator hands freed addresses to new tensors, so an address alone
# could return another weight's layout.
_RESIDENT_CACHE: "OrderedDict[tuple, _CacheEntry]" = OrderedDict()


class _CacheEntry:
    __slots__ = ("refs", "versions", "rw", "__weakref__")

    def __init__(self, tensors, rw):
        self.refs = tuple(weakref.ref(t) for t in tensors)
        self.versions = tuple(t._version for t in tensors)
        self.rw = rw

    def valid_for(self, tensors) -> bool:
        return all(r() is t and t._version == v for r, t, v in zip(self.refs, tensors, self.versions))


def _evict(key, ent_ref) -> None:
    if _RESIDENT_CACHE.get(key) is ent_ref():
        _RESIDENT_CACHE.pop(key, None)


def cached_resident(key_tag, streams, build) -> ResidentWeight:
    """The resident layout built by ``build()`` from the tensors ``streams``,
    reused while those very tensor objects live unmodified.  The lookup key
    holds their addresses; the entry is checked against the objects and their
    in-place version counters, so a new tensor at a freed address, or a stream
    edited in place, gets a fresh layout."""
    key = (key_tag,) + tuple(t.data_ptr() if t is not None else 0 for t in streams)
    live = tuple(t for t in streams if t is not None)
    ent = _RESIDENT_CACHE.get(key)
    if ent is not None and ent.valid_for(live):
        _RESIDENT_CACHE.move_to_end(key)
        return ent.rw
    ent = _CacheEntry(live, build())
    _RESIDENT_CACHE[key] = ent
    # the layout is released as soon as the first stream it came from dies
    weakref.finalize(live[0], _evict, key, weakref.ref(ent))
    while len(_RESIDENT_CACHE) > _CACHE_SLOTS:
        _RESIDENT_CACHE.popitem(last=False)
    return ent.rw


def _pad1(t: torch.Tensor) -> torch.Tensor:
    """One zero word appended, as the reference pads its streams (bf16x_fused.py:145-146)."""
    return torch.cat([t, torch.zeros(1, dtype=t.dtype, device=t.device)])


def csr_to_table(olk: torch.Tensor, old: torch.Tensor, oloff: torch.Tensor, in_f: int):
    """Per-row CSR (column, true delta, row offsets) -> the flat overflow table
    (ascending flat index int32, true delta uint8) that the decode and repack
    kernels read.  Inverse of the CSR build in bf16x_fused.py:165-179."""
    dev = olk.device
    counts = (oloff[1:].to(torch.int64) - oloff[:-1].to(torch.int64))
    rows = torch.repeat_interleave(torch.arange(counts.numel(), device=dev, dtype=torch.int64), counts)
    idx = rows * int(in_f) + olk.to(torch.int64)
    idx, order = torch.sort(idx, stable=True)
    val = old.to(torch.int64)[order]
    if idx.numel() and int(idx[-1]) >= 2**31:
        raise _lib.Bf16xError("overflow table index beyond int32 (out_f * in_f >= 2^31)")
    return idx.to(torch.int32), val.to(torch.uint8)


def _resident_from_streams(sign, mant, delta, emax, ovf_idx, ovf_val, out_f, in_f) -> ResidentWeight:
    p = {"sign_packed": sign, "mant_packed": mant, "delta_packed": delta, "emax": emax,
         "delta_ovf_idx": ovf_idx, "delta_ovf_val": ovf_val, "out_f": int(out_f), "in_f": int(in_f), "sub": 16}
    return ResidentWeight.from_packed(p, device=sign.device)


def clear_cache() -> None:
    """Drop the resident layouts built by ``bf16x_fused_gemv``.  Not needed
    for correctness: an entry is rebuilt whenever a stream tensor it was built
    from has died or been modified in place (torch's version counter); this
    only releases the device memory early."""
    _RESIDENT_CACHE.clear()


def bf16x_fused_gemv(x, sign, mant, delta, emax, olk, old, oloff,
                     out_f, in_f, group=16, r=4, bk=256, num_warps=2):
    """y[out_f] (bf16) = W x for one activation vector x[in_f], W given as
    flat streams + per-row overflow CSR (bf16x_fused.py:114-127).  Unlike the
    reference there is no ``in_f % bk == 0`` restriction."""
    _lib.require_cuda(x, "x")
    if group != 16:
        raise ValueError("only 16-element sub-blocks are supported")
    if x.numel() != in_f:
        raise ValueError(f"bf16x_fused_gemv takes one vector of {in_f} elements, got {x.numel()}")
    dev = x.device

    def build():
        oi, ov = csr_to_table(olk.to(dev), old.to(dev), oloff.to(dev), in_f)
        return _resident_from_streams(sign.to(dev), mant.to(dev), delta.to(dev), emax.to(dev), oi, ov,
                                      out_f, in_f)

    rw = cached_resident(("gemv", dev.index, int(out_f), int(in_f)), (sign, mant, delta, emax, olk, old, oloff),
                         build)
    return rw.gemv(x.reshape(1, in_f), out_dtype=torch.bfloat16).reshape(out_f)


# ------------------------------------------------------------------ #
#  shared decode buffer of the 'opt' mode (bf16x_fused.py:133-142):
#  one per process, reused by every layer, not thread-safe
# ------------------------------------------------------------------ #
_SHARED_DEC = None


def _shared_dec_buf(n: int, device) -> torch.Tensor:
    global _SHARED_DEC
    if _SHARED_DEC is None or _SHARED_DEC.numel() < n or _SHARED_DEC.device != torch.device(device):
        _SHARED_DEC = torch.empty(n, dtype=torch.bfloat16, device=device)
    return _SHARED_DEC


class Bf16xFused(nn.Module):
    """BF16X Linear with three forward modes (bf16x_fused.py:149-229).

    mode 'fused' (default): fused decode+GEMV / decode+GEMM kernels, W never
    materialised.  'opt': decode into the shared buffer, then F.linear.
    'repo': stand-alone decode with the overflow table on the host (copied per
    call, as the reference's as-is path does), then F.linear."""
    R, BK, WARPS = 4, 256, 2

    def __init__(self, packed: dict, bias: torch.Tensor | None = None, keep_cpu: bool = True):
        super().__init__()
        if not torch.cuda.is_available():
            raise _lib.Bf16xError("Bf16xFused runs on a CUDA device (bfloat16x_b200 has no CPU path)")
        self.out_features = int(packed["out_f"])
        self.in_features = int(packed["in_f"])
        self.N = self.out_features * self.in_features
        self.mode = "fused"
        dev = torch.device("cuda", torch.cuda.current_device())
        self._resident = ResidentWeight.from_packed(packed, device=dev)
        if keep_cpu:
            self._cpu = {k: packed[k] for k in ("sign_packed", "mant_packed", "delta_packed", "emax",
                                               "delta_ovf_idx", "delta_ovf_val")}
            self._dev_streams = {k: _pad1(packed[k].to(dev)) for k in ("sign_packed", "mant_packed",
                                                                      "delta_packed")}
            self._dev_streams["emax"] = packed["emax"].to(dev)
        else:
            self._cpu = None
            self._dev_streams = None
        if bias is not None:
            self.register_buffer("_bias", bias.detach().clone().to(dev))
        else:
            self._bias = None

    @property
    def resident(self) -> ResidentWeight:
        return self._resident

    def _decode_opt(self) -> torch.Tensor:
        buf = _shared_dec_buf(self.N, self._resident.device)[: self.N]
        return self._resident.decode(out=buf.view(self.out_features, self.in_features))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(x, "x")
        if self.mode == "fused":
            b = None if self._bias is None else self._bias
            od = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16
            return self._resident.linear(x, b, out_dtype=od).to(x.dtype)
        if self.mode == "repo" and self._cpu is not None:
            s = self._dev_streams
            w = bf16x_decode_triton(s["sign_packed"], s["mant_packed"], s["delta_packed"], s["emax"],
                                    self.out_features, self.in_features,
                                    self._cpu["delta_ovf_idx"], self._cpu["delta_ovf_val"], 16)
            return F.linear(x, w.to(x.dtype), None if self._bias is None else self._bias.to(x.dtype))
        w = self._decode_opt()
        return F.linear(x, w.to(x.dtype), None if self._bias is None else self._bias.to(x.dtype))


def _packed_bytes(p: dict) -> int:
    # the reference's byte count (bf16x_fused.py:254-256)
    return (p["sign_packed"].numel() * 4 + p["mant_packed"].numel() * 4 + p["delta_packed"].numel() * 4
            + p["emax"].numel() + p["delta_ovf_idx"].numel() * 5)


def _linear_targets(model: nn.Module, min_numel: int, skip):
    out = []
    for name, mod in model.named_modules():
        if not isinstance(mod, nn.Linear) or mod.weight.numel() < min_numel:
            continue
        if any(s in name for s in skip):
            continue
        out.append((name, mod))
    return out


def _set_module(model: nn.Module, name: str, new: nn.Module) -> None:
    parts = name.split(".")
    parent = model
    for q in parts[:-1]:
        parent = getattr(parent, q)
    setattr(parent, parts[-1], new)


@torch.no_grad()
def deploy_bf16x_fused(model: nn.Module, verbose: bool = True, skip=("lm_head", "embed"),
                       min_numel: int = 1000):
    """Replace every nn.Linear of at least ``min_numel`` weights whose name
    contains none of ``skip`` by a Bf16xFused layer (bf16x_fused.py:232-263).
    ``skip=()`` also packs lm_head.  Returns (packed bytes, weights)."""
    from .opqk_linear import bf16x_quantize
    targets = _linear_targets(model, min_numel, skip)
    total = n_el = 0
    for name, mod in targets:
        w = mod.weight.data
        p = bf16x_quantize(w.to(torch.bfloat16), sub=16)
        bias = mod.bias.data if mod.bias is not None else None
        _set_module(model, name, Bf16xFused(p, bias=bias))
        total += _packed_bytes(p)
        n_el += w.numel()
        mod.weight.data = torch.empty(0)
        del w, p
    if verbose:
        print(f"[bf16x-fused] {len(targets)} layers | {total/1e6:.0f}MB packed "
              f"({n_el*2/max(total, 1):.2f}x) | bpw={total*8/max(n_el, 1):.2f}", flush=True)
    return total, n_el


__all__ = ["bf16x_fused_gemv", "Bf16xFused", "deploy_bf16x_fused", "csr_to_table", "clear_cache"]
