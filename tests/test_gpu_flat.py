"""GPU parity of the flat-stream kernels: the fused decode (bf16x_decode_triton)
and the GPU packer (bf16x_quantize), both bit-exact against the reference's
golden vectors and the CPU oracle."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200.bf16x_decode import bf16x_decode_triton
from bfloat16x_b200.opqk_linear import bf16x_quantize
from bfloat16x_b200.synthetic import synthetic_weight
from oracle import oracle
from tests.gpu_util import GOLD, KEYS, bits_of, bf16_from_bits, dict_from_npz, load_flat, oracle_dict

pytestmark = pytest.mark.gpu
FLAT = load_flat()
CASES = list(FLAT["cases"])


def _decode(p, pad=False, ovf_device="cuda"):
    def s(k):
        t = p[k].cuda()
        if pad:
            t = torch.cat([t, torch.zeros(1, dtype=t.dtype, device=t.device)])
        return t
    oi = p["delta_ovf_idx"].to(ovf_device)
    ov = p["delta_ovf_val"].to(ovf_device)
    out = bf16x_decode_triton(s("sign_packed"), s("mant_packed"), s("delta_packed"), p["emax"].cuda(),
                              p["out_f"], p["in_f"], oi, ov, 16)
    torch.cuda.synchronize()
    return bits_of(out)


@pytest.mark.parametrize("case", CASES)
def test_decode_matches_reference(case):
    p = dict_from_npz(FLAT, case)
    ref = FLAT[f"{case}/decoded"]
    assert np.array_equal(_decode(p), ref)
    assert np.array_equal(_decode(p, pad=True), ref)       # _pad1-style streams
    assert np.array_equal(_decode(p, ovf_device="cpu"), ref)  # table on the host, as in the reference API
    _lib.check_device_status()


def test_decode_filtered_table():
    # the reference's GPU paths keep only entries with delta > 7 (bf16x_triton_test.py:96)
    w = bits_of(synthetic_weight(257, 320, seed=3))
    p = oracle_dict(w)
    keep = p["delta_ovf_val"] > 7
    p["delta_ovf_idx"], p["delta_ovf_val"] = p["delta_ovf_idx"][keep], p["delta_ovf_val"][keep]
    assert np.array_equal(_decode(p), w)


@pytest.mark.parametrize("shape", [(2048, 1536), (4099, 333), (1, 8193), (3, 5)])
def test_decode_vs_oracle(shape):
    w = bits_of(synthetic_weight(*shape, seed=11))
    p = oracle_dict(w)
    got = _decode(p)
    assert np.array_equal(got, oracle.decode({k: v.numpy() if torch.is_tensor(v) else v for k, v in p.items()}))
    assert np.array_equal(got, w)


def test_decode_dense_overflow_and_many_tiles():
    """Tiles with far more overflow entries than the kernel requests ahead
    (magnitudes spread over 2^-40..2^0: most weights overflow), and enough
    tiles that every persistent CTA walks several."""
    from tests.test_gpu_gemm import _dense_patch_weight
    w = _dense_patch_weight(600, 1024, seed=13)
    p = oracle_dict(w)
    assert p["delta_ovf_idx"].numel() > 600 * 1024 // 2
    assert np.array_equal(_decode(p), w)
    w2 = synthetic_weight(4096, 4096, seed=17, device="cuda")
    p2 = bf16x_quantize(w2, device="cuda")
    out = bf16x_decode_triton(p2["sign_packed"], p2["mant_packed"], p2["delta_packed"], p2["emax"], 4096, 4096,
                              p2["delta_ovf_idx"], p2["delta_ovf_val"])
    assert torch.equal(out.view(torch.int16), w2.view(torch.int16))
    _lib.check_device_status()


def test_decode_unaligned_streams():
    """Streams that do not start on a 16-byte boundary take plain loads
    instead of the bulk copies; the result is the same."""
    w = bits_of(synthetic_weight(1000, 1536, seed=19))
    p = oracle_dict(w)

    def shifted(t):
        buf = torch.zeros(t.numel() + 4, dtype=t.dtype, device="cuda")
        buf[1:1 + t.numel()] = t.cuda()
        return buf[1:1 + t.numel()]
    s, m, d = (shifted(p[k]) for k in ("sign_packed", "mant_packed", "delta_packed"))
    e = shifted(p["emax"])
    assert s.data_ptr() % 16 != 0 and e.data_ptr() % 16 != 0
    out = bf16x_decode_triton(s, m, d, e, 1000, 1536, p["delta_ovf_idx"], p["delta_ovf_val"])
    assert np.array_equal(bits_of(out), w)
    _lib.check_device_status()


def test_decode_reports_unsorted_table():
    w = bits_of(synthetic_weight(64, 512, seed=5))
    p = oracle_dict(w)
    assert p["delta_ovf_idx"].numel() > 4
    idx = p["delta_ovf_idx"].clone()
    idx[[1, 2]] = idx[[2, 1]]
    p["delta_ovf_idx"] = idx
    _lib.device_status()  # clear
    _decode(p)
    flags = _lib.device_status()
    assert flags & 2, flags
    assert _lib.device_status() == 0   # read clears


@pytest.mark.parametrize("case", CASES)
def test_quantize_matches_reference(case):
    w = FLAT[f"{case}/w"]
    p = bf16x_quantize(bf16_from_bits(w, "cuda"))
    assert p["out_f"] == w.shape[0] and p["in_f"] == w.shape[1] and p["sub"] == 16
    for k in KEYS:
        ref = FLAT[f"{case}/{k}"]
        got = p[k].numpy()
        assert p[k].device.type == "cpu"
        assert got.dtype == ref.dtype and got.shape == ref.shape, (k, got.dtype, got.shape, ref.shape)
        assert np.array_equal(got, ref), k


def test_quantize_config1_hashes():
    h = json.load(open(os.path.join(GOLD, "golden_hashes.json")))["config1_2048x1536"]
    p = bf16x_quantize(synthetic_weight(2048, 1536, seed=0).cuda())
    for k in KEYS:
        assert hashlib.sha256(p[k].numpy().tobytes()).hexdigest() == h[k], k
    assert p["delta_ovf_idx"].numel() == h["n_ovf"]


@pytest.mark.parametrize("shape", [(4096, 4096), (333, 4099), (1, 1)])
def test_quantize_vs_oracle(shape):
    w = synthetic_weight(*shape, seed=21)
    p = bf16x_quantize(w.cuda())
    q = oracle.quantize(bits_of(w), *shape)
    for k in KEYS:
        assert np.array_equal(p[k].numpy(), q[k].view(p[k].numpy().dtype)), k
