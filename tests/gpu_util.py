"""Shared helpers of the GPU parity tests (oracle-side conversions)."""
import os

import numpy as np
import torch

from oracle import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KEYS = ("emax", "sign_packed", "mant_packed", "delta_packed", "delta_ovf_idx", "delta_ovf_val")


def load_flat():
    return np.load(os.path.join(GOLD, "flat_small.npz"))


def bits_of(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 numpy bit patterns."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bf16_from_bits(b: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16).to(device)


def dict_from_npz(npz, case) -> dict:
    w = npz[f"{case}/w"]
    p = {k: torch.from_numpy(np.ascontiguousarray(npz[f"{case}/{k}"])) for k in KEYS}
    p.update(out_f=w.shape[0], in_f=w.shape[1], sub=16)
    return p


def oracle_dict(bits: np.ndarray) -> dict:
    p = oracle.quantize(bits, *bits.shape)
    q = {k: torch.from_numpy(np.ascontiguousarray(p[k])) for k in KEYS}
    q.update(out_f=bits.shape[0], in_f=bits.shape[1], sub=16)
    return q


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
