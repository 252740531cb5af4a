"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference project (dfytensor/bfloat16x) is
importable, e.g. ``python tests/golden/make_golden.py /path/to/reference``.
The outputs (``flat_small.npz``, ``gguf_small.npz``, ``golden_hashes.json``)
are committed; tests read only those files and never the reference itself.

What is recorded, all produced by the REFERENCE's own functions:
* ``bf16x_quantize`` (opqk_linear.py:291-324) dicts for small seeded shapes,
  including ragged N (not a multiple of 16 or 32), all-zero, subnormal,
  inf/NaN and huge-outlier weights;
* ``BF16XLinear._decode_tile`` (opqk_linear.py:360-377) outputs;
* the decoded-bf16 fp32-accumulate matmul ``x.float() @ W.float().T``
  (the GEMV/GEMM parity target) for a few batches;
* ``bf16x_gguf_block`` quantize/dequantize/pack_ovf outputs
  (bf16x_gguf_block.py:44-187) for small shapes and SHA-256 digests for the
  reference's own self-test shapes (bf16x_gguf_block.py:196-232);
* SHA-256 digests of every stream of the 2048x1536 CPU-plumbing config.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root

from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight  # noqa: E402


def _sha(a) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


def special_weights() -> dict:
    """Hand-made weights covering the format's edge cases (as bf16 bit patterns)."""
    out = {}
    out["zeros_4x16"] = np.zeros((4, 16), np.uint16)
    # subnormals (exponent field 0), signed zeros, +-inf, NaN, max finite
    rng = np.random.default_rng(7)
    b = rng.integers(0, 1 << 16, size=(8, 64), dtype=np.uint64).astype(np.uint16)
    b[0, :16] = rng.integers(0, 128, 16).astype(np.uint16)            # subnormals
    b[1, :4] = [0x0000, 0x8000, 0x7F80, 0xFF80]                        # +-0, +-inf
    b[1, 4:8] = [0x7FC0, 0xFFC1, 0x7F7F, 0x0001]                        # NaNs, max, min sub
    b[2, :] = 0x3F80                                                   # all ones
    b[3, ::5] = 0x7F00                                                 # huge outliers
    out["special_8x64"] = b
    # one huge element per sub-block: deltas up to 254
    c = np.full((2, 48), 0x0081, np.uint16)
    c[:, ::16] = 0x7F7F
    out["spread_2x48"] = c
    return out


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from opqk_linear import BF16XLinear, bf16x_quantize  # reference code
    import bf16x_gguf_block as gg                        # reference code

    torch.manual_seed(0)
    flat = {}
    cases = []
    shapes = [(3, 5), (1, 1), (1, 33), (4, 48), (16, 256), (33, 96), (64, 512), (24, 1536)]
    weights = {f"syn_{o}x{i}": synthetic_weight(o, i, seed=o * 1000 + i).view(torch.int16)
               .numpy().view(np.uint16) for o, i in shapes}
    weights.update(special_weights())
    for name, bits in weights.items():
        o, i = bits.shape
        w = torch.from_numpy(bits.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)
        p = bf16x_quantize(w, sub=16)
        dec = BF16XLinear.from_packed(p)._decode_tile(0, o).view(torch.int16).numpy().view(np.uint16)
        flat[f"{name}/w"] = bits
        for k in ("emax", "sign_packed", "mant_packed", "delta_packed", "delta_ovf_idx", "delta_ovf_val"):
            flat[f"{name}/{k}"] = p[k].numpy()
        flat[f"{name}/decoded"] = dec
        finite = np.isfinite((dec.astype(np.uint32) << 16).view(np.float32)).all()
        if finite:
            for bsz in (1, 3, 8):
                x = synthetic_activation(bsz, i, seed=bsz)
                y = (x.float() @ torch.from_numpy(dec.view(np.int16).copy()).view(torch.bfloat16).float().T)
                flat[f"{name}/x{bsz}"] = x.view(torch.int16).numpy().view(np.uint16)
                flat[f"{name}/y{bsz}"] = y.numpy()
        cases.append(name)
    flat["cases"] = np.array(cases)
    np.savez_compressed(os.path.join(HERE, "flat_small.npz"), **flat)

    # ---- GGUF blocks --------------------------------------------------------
    gguf = {}
    gcases = []
    rng = np.random.default_rng(0)
    gshapes = [(4, 64), (8, 96), (3, 32)]
    for shape in gshapes:
        w = (rng.standard_normal(shape) * 0.13).astype(np.float32)
        idx = rng.choice(w.size, max(1, w.size // 50), replace=False)
        w.reshape(-1)[idx] *= rng.standard_normal(len(idx)) * 64
        name = f"g_{shape[0]}x{shape[1]}"
        gcases.append(name)
        packed = gg.quantize_tensor(w)
        gguf[f"{name}/x"] = w
        gguf[f"{name}/blocks"] = packed
        gguf[f"{name}/deq"] = gg.dequantize_blocks(packed)
        blob = gg.pack_ovf(w)
        gguf[f"{name}/ovf"] = np.frombuffer(blob, np.uint8)
        gguf[f"{name}/lossless"] = gg.dequantize_lossless(packed, blob)
        gguf[f"{name}/bf16bits"] = gg.fp32_to_bf16_bits(w)
    # the special bit patterns through the GGUF path (bf16-exact inputs)
    sp = special_weights()["special_8x64"]
    spf = (sp.astype(np.uint32) << 16).view(np.float32)
    gguf["g_special/x"] = spf
    gguf["g_special/blocks"] = gg.quantize_tensor(spf)
    gguf["g_special/deq"] = gg.dequantize_blocks(gguf["g_special/blocks"])
    gguf["g_special/ovf"] = np.frombuffer(gg.pack_ovf(spf, bf16_exact=True), np.uint8)
    gcases.append("g_special")
    gguf["cases"] = np.array(gcases)
    np.savez_compressed(os.path.join(HERE, "gguf_small.npz"), **gguf)

    # ---- digests of larger reference outputs --------------------------------
    hashes = {}
    w = synthetic_weight(2048, 1536, seed=0)
    p = bf16x_quantize(w, sub=16)
    dec = BF16XLinear.from_packed(p)._decode_tile(0, 2048)
    hashes["config1_2048x1536"] = {
        "recipe": "synthetic_weight(2048, 1536, seed=0)",
        "w": _sha(w.view(torch.int16).numpy()),
        **{k: _sha(p[k].numpy()) for k in ("emax", "sign_packed", "mant_packed", "delta_packed",
                                            "delta_ovf_idx", "delta_ovf_val")},
        "n_ovf": int(p["delta_ovf_idx"].numel()),
        "n_ovf_gt7": int((p["delta_ovf_val"] > 7).sum()),
        "decoded_equals_input": bool((dec.view(torch.int16) == w.view(torch.int16)).all()),
    }
    x = synthetic_activation(1, 1536, seed=1)
    y = (x.float() @ dec.float().T).numpy()
    np.save(os.path.join(HERE, "config1_y1.npy"), y.astype(np.float32))
    hashes["config1_2048x1536"]["x_recipe"] = "synthetic_activation(1, 1536, seed=1)"
    # the reference GGUF self-test shapes and input recipe (bf16x_gguf_block.py:203-207)
    rng = np.random.default_rng(0)
    for shape in [(256, 512), (300, 576), (1024, 2048)]:
        w = (rng.standard_normal(shape) * 0.13).astype(np.float32)
        idx = rng.choice(w.size, w.size // 200, replace=False)
        w.reshape(-1)[idx] *= rng.standard_normal(len(idx)) * 8
        packed = gg.quantize_tensor(w)
        blob = gg.pack_ovf(w)
        hashes[f"gguf_selftest_{shape[0]}x{shape[1]}"] = {
            "x": _sha(w), "blocks": _sha(packed), "deq": _sha(gg.dequantize_blocks(packed)),
            "ovf": hashlib.sha256(blob).hexdigest(), "n_ovf": int(gg.ovf_stats(w)[0]),
        }
    with open(os.path.join(HERE, "golden_hashes.json"), "w") as f:
        json.dump(hashes, f, indent=1, sort_keys=True)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.basename(__file__)} <path of the reference checkout>")
    main(sys.argv[1])
