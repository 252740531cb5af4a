"""Drop-in for the reference's ``pack_to_disk`` module (pack_to_disk.py): the
on-disk "bf16x-v1" format and a loader that feeds it to the device repack.

The files are the reference's, byte for byte (pack_to_disk.py:10-22):

* ``<prefix>.safetensors`` (metadata ``{"format": "bf16x"}``), per packed
  linear ``<name>``: ``.sign`` / ``.mant`` / ``.delta`` int32 bit-stream
  words with one zero word appended, ``.emax`` uint8 (one per 16 elements),
  ``.ovf_i`` int64 flat index / ``.ovf_v`` int32 true delta of the overflow
  entries whose delta exceeds 7 (a stored 7 with no entry stays 7), and
  ``.bias`` bf16 when the layer has one;
* ``<prefix>.meta.json``: ``{"kind": "bf16x-v1", "tensors": {name: {sign,
  mant, delta, emax, ovf_i, ovf_v, out_f, in_f, N, n_fix[, bias]}}}`` where
  the six stream fields name the tensors above.

``pack_model_to_disk`` quantises every selected ``nn.Linear`` with the GPU
packer (``bf16x_quantize``), writes the two files and drops each original
weight as soon as it is packed.  ``replace_linears_from_packed`` maps the
blob (safetensors mmap), copies each layer's flat streams to the GPU and
builds the resident layout there with the device repack -- no
re-quantisation -- then swaps the layer for a ``Bf16xStreamLinear``, which
runs the fused decode+GEMV (up to 16 rows) or decode+GEMM (more rows) on the
exact weights.  ``resident=False`` keeps the resident layout in pinned host
memory and stages it to the device on every forward, as ``Bf16xGemmLinear``
does.
"""
from __future__ import annotations

import json
import os
import time

import torch
import torch.nn as nn

from . import _lib
from .bf16x_fused import _linear_targets, _pad1, _set_module
from .bf16x_gemm_fused import Bf16xGemmLinear

KIND = "bf16x-v1"
_DEFAULT_SKIP = ("embed", "lm_head")
_STREAMS = ("sign", "mant", "delta", "emax", "ovf_i", "ovf_v")


def disk_tensors(p: dict, bias: torch.Tensor | None = None) -> dict:
    """The on-disk tensors of one packed linear, keyed by field name: the
    bf16x_quantize dict ``p`` with its streams padded by one word and its
    overflow table reduced to the entries with delta > 7
    (pack_to_disk.py:62-76)."""
    oi = torch.as_tensor(p["delta_ovf_idx"]).cpu().to(torch.int64)
    ov = torch.as_tensor(p["delta_ovf_val"]).cpu().to(torch.int64)
    keep = ov > 7
    out = {
        "sign": _pad1(torch.as_tensor(p["sign_packed"]).cpu().to(torch.int32)),
        "mant": _pad1(torch.as_tensor(p["mant_packed"]).cpu().to(torch.int32)),
        "delta": _pad1(torch.as_tensor(p["delta_packed"]).cpu().to(torch.int32)),
        "emax": torch.as_tensor(p["emax"]).cpu().to(torch.uint8),
        "ovf_i": oi[keep],
        "ovf_v": ov[keep].to(torch.int32),
    }
    if bias is not None:
        out["bias"] = bias.detach().to(torch.bfloat16).cpu()
    return {k: v.contiguous() for k, v in out.items()}


class _Writer:
    """Collects layers for one bf16x-v1 blob and writes the two files."""

    def __init__(self):
        self.blobs: dict = {}
        self.meta = {"kind": KIND, "tensors": {}}
        self.total = 0

    def add(self, name: str, p: dict, bias: torch.Tensor | None = None) -> None:
        t = disk_tensors(p, bias)
        m = {}
        for key, val in t.items():
            gk = f"{name}.{key}"
            self.blobs[gk] = val
            self.total += val.numel() * val.element_size()
            m[key] = gk
        m["out_f"], m["in_f"] = int(p["out_f"]), int(p["in_f"])
        m["N"] = int(p["out_f"]) * int(p["in_f"])
        m["n_fix"] = int(t["ovf_i"].numel())
        # the reference writes the bias name last
        if "bias" in m:
            m["bias"] = m.pop("bias")
        self.meta["tensors"][name] = m

    def save(self, out_prefix: str) -> None:
        from safetensors.torch import save_file
        save_file(self.blobs, out_prefix + ".safetensors", metadata={"format": "bf16x"})
        with open(out_prefix + ".meta.json", "w") as f:
            json.dump(self.meta, f)


def write_bf16x_v1(out_prefix: str, layers) -> int:
    """Write ``layers`` (iterable of (name, bf16x_quantize dict, bias or
    None)) as ``<out_prefix>.safetensors`` + ``.meta.json``.  Returns the
    bytes of tensor data written."""
    w = _Writer()
    for name, p, bias in layers:
        w.add(name, p, bias)
    w.save(out_prefix)
    return w.total


@torch.no_grad()
def pack_model_to_disk(model: nn.Module, out_prefix: str, min_numel: int = 4096, sub: int = 16,
                       skip=_DEFAULT_SKIP, verbose: bool = True):
    """Pack every nn.Linear with at least ``min_numel`` weights and a name
    containing none of ``skip`` into the bf16x-v1 files (pack_to_disk.py:40-105).
    Packed layers lose their weight (and bias) tensors; the rest of the model
    is untouched.  Returns (n_packed, packed_bytes)."""
    from .opqk_linear import bf16x_quantize
    w = _Writer()
    t0 = time.time()
    n = 0
    for name, mod in _linear_targets(model, min_numel, skip):
        p = bf16x_quantize(mod.weight.data.detach().to(torch.bfloat16), sub=sub)
        w.add(name, p, mod.bias.data if mod.bias is not None else None)
        if mod.bias is not None:
            mod.bias.data = torch.empty(0)
        mod.weight.data = torch.empty(0)
        del p
        n += 1
        if verbose and n % 50 == 0:
            print(f"  {n} packed, blob {w.total/1e9:.1f}GB, {time.time()-t0:.0f}s", flush=True)
    if verbose:
        print(f"saving {n} packed linears ({w.total/1e9:.2f}GB) ...", flush=True)
    w.save(out_prefix)
    if verbose:
        print(f"  -> {out_prefix}.safetensors ({os.path.getsize(out_prefix + '.safetensors')/1e9:.2f}GB)", flush=True)
    return n, w.total


def read_meta(out_prefix: str) -> dict:
    """The ``tensors`` table of ``<out_prefix>.meta.json`` (kind checked)."""
    with open(out_prefix + ".meta.json") as f:
        meta = json.load(f)
    if meta.get("kind") != KIND:
        raise _lib.Bf16xError(f"{out_prefix}.meta.json: kind {meta.get('kind')!r}, expected {KIND!r}")
    return meta["tensors"]


def blob_to_packed(entry: dict, blob: dict) -> dict:
    """A bf16x_quantize-style dict over one layer's on-disk tensors (no copy
    of the streams; the overflow table converted to the C-ABI types)."""
    oi = blob.get("ovf_i")
    ov = blob.get("ovf_v")
    if oi is None or oi.numel() == 0:
        oi = torch.zeros(0, dtype=torch.int32)
        ov = torch.zeros(0, dtype=torch.uint8)
    else:
        if int(oi.max()) >= 2 ** 31 or int(oi.min()) < 0:
            raise _lib.Bf16xError("overflow index outside the 32-bit range of the device table")
        if int(ov.min()) < 0 or int(ov.max()) > 255:
            raise _lib.Bf16xError("overflow delta outside 0..255")
        oi = oi.to(torch.int32)
        ov = ov.to(torch.uint8)
    return {"sign_packed": blob["sign"], "mant_packed": blob["mant"], "delta_packed": blob["delta"],
            "emax": blob["emax"], "delta_ovf_idx": oi, "delta_ovf_val": ov,
            "out_f": int(entry["out_f"]), "in_f": int(entry["in_f"]), "sub": 16}


class Bf16xStreamLinear(Bf16xGemmLinear):
    """A packed linear fed from the bf16x-v1 blob (pack_to_disk.py:108-224).

    resident=True : the resident layout lives in HBM (built once from the
                    flat streams by the device repack).
    resident=False: it lives in pinned host memory and is staged to the
                    device on every forward."""

    def __init__(self):
        raise RuntimeError("use from_packed()")

    @classmethod
    def from_packed(cls, entry: dict, blob: dict, resident: bool = True) -> "Bf16xStreamLinear":
        obj = cls.__new__(cls)
        bias = blob.get("bias") if entry.get("bias") else None
        Bf16xGemmLinear.__init__(obj, blob_to_packed(entry, blob), bias=bias, resident=resident)
        obj.N = int(entry["N"])
        obj.n_fix = int(entry.get("n_fix", 0))
        return obj

    @property
    def bias(self):
        return self._bias


@torch.no_grad()
def replace_linears_from_packed(model: nn.Module, out_prefix: str, resident_fn=None,
                                keep_rest_bf16: bool = True, verbose: bool = True) -> int:
    """Swap every nn.Linear named in ``<out_prefix>.meta.json`` for a
    Bf16xStreamLinear built from the mmapped blob (pack_to_disk.py:227-265).
    ``resident_fn(name) -> bool`` picks HBM-resident or pinned-host per layer
    (default: resident).  Linears not in the blob are cast to bf16 when
    ``keep_rest_bf16``.  The model is then moved to the GPU.  Returns the
    number of layers replaced."""
    from safetensors import safe_open
    if not torch.cuda.is_available():
        raise _lib.Bf16xError("replace_linears_from_packed builds the layers on a CUDA device")
    meta = read_meta(out_prefix)
    n = n_res = n_dma = 0
    t0 = time.time()
    with safe_open(out_prefix + ".safetensors", framework="pt", device="cpu") as sf:
        for name, mod in list(model.named_modules()):
            if not isinstance(mod, nn.Linear):
                continue
            if name in meta:
                entry = meta[name]
                keys = _STREAMS + (("bias",) if entry.get("bias") else ())
                blob = {k: sf.get_tensor(entry[k]) for k in keys if entry.get(k)}
                res = resident_fn(name) if resident_fn else True
                _set_module(model, name, Bf16xStreamLinear.from_packed(entry, blob, resident=res))
                mod.weight.data = torch.empty(0)
                n += 1
                n_res += int(res)
                n_dma += int(not res)
                del blob
            elif keep_rest_bf16:
                mod.weight.data = mod.weight.data.to(torch.bfloat16)
    model.cuda()
    torch.cuda.empty_cache()
    if verbose:
        print(f"[bf16x] {n} linears from disk in {time.time()-t0:.0f}s | {n_res} resident + {n_dma} DMA",
              flush=True)
    return n


__all__ = ["KIND", "disk_tensors", "write_bf16x_v1", "pack_model_to_disk", "read_meta", "blob_to_packed",
           "Bf16xStreamLinear", "replace_linears_from_packed"]
