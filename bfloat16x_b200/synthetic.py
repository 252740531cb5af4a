"""Seeded synthetic inputs with the benchmark distributions.

No checkpoint or dataset is available offline, so every benchmark and test
draws its weights and activations from these generators:

* weights: N(0, 0.02), then 0.5% of the entries (a seeded permutation) are
  multiplied by 2**k with k uniform in 4..8, which forces exponent deltas of
  7 and more (the overflow side table) -- the recipe of the benchmark configs;
* activations: bf16 N(0, 1) from a separate seed.
"""
from __future__ import annotations

import torch


def synthetic_weight(out_f: int, in_f: int, seed: int = 0, device="cpu",
                     std: float = 0.02, outlier_frac: float = 0.005) -> torch.Tensor:
    """bf16 [out_f, in_f] weight with the overflow-forcing outliers."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(out_f, in_f, generator=g, device=device, dtype=torch.float32) * std
    n = w.numel()
    k = int(n * outlier_frac)
    if k:
        idx = torch.randperm(n, generator=g, device=device)[:k]
        e = torch.randint(4, 9, (k,), generator=g, device=device).to(torch.float32)
        w.view(-1)[idx] *= torch.exp2(e)
    return w.to(torch.bfloat16)


def synthetic_activation(batch: int, in_f: int, seed: int = 1, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(batch, in_f, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
