"""Generate the on-disk "bf16x-v1" fixture with the REFERENCE's own packer.

Run where the reference project (dfytensor/bfloat16x) is importable:
``python tests/golden/make_disk_golden.py /path/to/reference``.  It builds a
small seeded model, packs it with the reference's ``pack_model_to_disk``
(pack_to_disk.py:40-105) and writes, next to this script:

* ``disk_v1_small.safetensors`` / ``disk_v1_small.meta.json`` -- the files
  exactly as the reference writes them;
* ``disk_v1_small_weights.npz`` -- the original bf16 weights (uint16 bits)
  and biases of every module, so a loader can be checked bit for bit.

Tests read only these files, never the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root

from bfloat16x_b200.synthetic import synthetic_weight  # noqa: E402


class TinyModel(nn.Module):
    """Linears with and without bias, one below the size threshold, one
    ragged (in_f not a multiple of 16) and an lm_head (skipped by default)."""

    def __init__(self):
        super().__init__()
        self.up = nn.Linear(96, 80, bias=True)
        self.down = nn.Linear(80, 300, bias=False)
        self.ragged = nn.Linear(75, 112, bias=True)
        self.small = nn.Linear(16, 16, bias=False)
        self.lm_head = nn.Linear(300, 128, bias=False)


def build_model() -> TinyModel:
    torch.manual_seed(0)
    m = TinyModel()
    for i, (name, mod) in enumerate(m.named_modules()):
        if isinstance(mod, nn.Linear):
            w = synthetic_weight(mod.out_features, mod.in_features, seed=100 + i)
            mod.weight.data = w.to(torch.bfloat16)
            if mod.bias is not None:
                g = torch.Generator().manual_seed(200 + i)
                mod.bias.data = (torch.randn(mod.out_features, generator=g) * 0.1).to(torch.bfloat16)
    return m


def main(ref_dir: str) -> None:
    sys.path.insert(0, ref_dir)
    from pack_to_disk import pack_model_to_disk  # the reference's packer

    m = build_model()
    arrays = {}
    for name, mod in m.named_modules():
        if isinstance(mod, nn.Linear):
            arrays[f"{name}.weight"] = mod.weight.data.view(torch.int16).numpy().view(np.uint16).copy()
            if mod.bias is not None:
                arrays[f"{name}.bias"] = mod.bias.data.view(torch.int16).numpy().view(np.uint16).copy()
    np.savez_compressed(os.path.join(HERE, "disk_v1_small_weights.npz"), **arrays)
    n, total = pack_model_to_disk(m, os.path.join(HERE, "disk_v1_small"), verbose=False)
    print(f"packed {n} linears, {total} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.basename(__file__)} <path of the reference checkout>")
    main(sys.argv[1])
