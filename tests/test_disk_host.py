"""The on-disk bf16x-v1 format on the host: the committed fixture written by
the reference's own packer (tests/golden/make_disk_golden.py) is read, pinned
to the original weights with the CPU oracle, and reproduced byte for byte by
this package's writer from oracle-packed dicts."""
import json
import os

import numpy as np
import torch
from safetensors import safe_open

from bfloat16x_b200 import pack_to_disk as ptd
from oracle import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")
PREFIX = os.path.join(GOLD, "disk_v1_small")
PACKED = ("up", "down", "ragged")          # small (256 weights) and lm_head are not packed


def _weights():
    return dict(np.load(os.path.join(GOLD, "disk_v1_small_weights.npz")))


def _fixture_tensors():
    with safe_open(PREFIX + ".safetensors", framework="pt", device="cpu") as f:
        return {k: f.get_tensor(k) for k in f.keys()}, f.metadata()


def test_meta_matches_reference_layout():
    meta = ptd.read_meta(PREFIX)
    assert sorted(meta) == sorted(PACKED)
    w = _weights()
    for name in PACKED:
        e = meta[name]
        out_f, in_f = w[f"{name}.weight"].shape
        assert (e["out_f"], e["in_f"], e["N"]) == (out_f, in_f, out_f * in_f)
        assert ("bias" in e) == (f"{name}.bias" in w)


def test_fixture_streams_decode_to_the_weights():
    # pins the fixture: the oracle decode of its streams is the original bf16
    meta = ptd.read_meta(PREFIX)
    t, md = _fixture_tensors()
    assert md == {"format": "bf16x"}
    w = _weights()
    for name in PACKED:
        e = meta[name]
        p = ptd.blob_to_packed(e, {k: t[e[k]] for k in ptd._STREAMS})
        assert p["delta_ovf_val"].numel() == e["n_fix"] and bool((p["delta_ovf_val"] > 7).all())
        dec = oracle.decode_scatter({k: (v.numpy() if torch.is_tensor(v) else v) for k, v in p.items()})
        assert np.array_equal(dec, w[f"{name}.weight"])
        if "bias" in e:
            assert np.array_equal(t[e["bias"]].view(torch.int16).numpy().view(np.uint16), w[f"{name}.bias"])


def test_writer_reproduces_reference_files(tmp_path):
    w = _weights()
    layers = []
    for name in PACKED:
        bits = w[f"{name}.weight"]
        p = oracle.quantize(bits, *bits.shape)
        p = {k: (torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else v) for k, v in p.items()}
        b = w.get(f"{name}.bias")
        bias = None if b is None else torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16)
        layers.append((name, p, bias))
    out = str(tmp_path / "mine")
    total = ptd.write_bf16x_v1(out, layers)
    ref_t, _ = _fixture_tensors()
    assert total == sum(v.numel() * v.element_size() for v in ref_t.values())
    with open(out + ".meta.json") as f, open(PREFIX + ".meta.json") as g:
        assert f.read() == g.read()
    with open(out + ".safetensors", "rb") as f, open(PREFIX + ".safetensors", "rb") as g:
        assert f.read() == g.read()


def test_overflow_table_conversion_and_guards():
    e = {"out_f": 2, "in_f": 16, "N": 32}
    blob = {"sign": torch.zeros(2, dtype=torch.int32), "mant": torch.zeros(8, dtype=torch.int32),
            "delta": torch.zeros(4, dtype=torch.int32), "emax": torch.zeros(2, dtype=torch.uint8),
            "ovf_i": torch.tensor([3, 9], dtype=torch.int64), "ovf_v": torch.tensor([8, 30], dtype=torch.int32)}
    p = ptd.blob_to_packed(e, blob)
    assert p["delta_ovf_idx"].dtype == torch.int32 and p["delta_ovf_val"].dtype == torch.uint8
    assert p["delta_ovf_idx"].tolist() == [3, 9] and p["delta_ovf_val"].tolist() == [8, 30]
    blob["ovf_i"] = torch.tensor([2 ** 31], dtype=torch.int64)
    blob["ovf_v"] = torch.tensor([8], dtype=torch.int32)
    try:
        ptd.blob_to_packed(e, blob)
    except RuntimeError as err:
        assert "32-bit" in str(err)
    else:
        raise AssertionError("index >= 2^31 accepted")


def test_read_meta_rejects_other_kinds(tmp_path):
    p = str(tmp_path / "x")
    with open(p + ".meta.json", "w") as f:
        json.dump({"kind": "other", "tensors": {}}, f)
    try:
        ptd.read_meta(p)
    except RuntimeError as err:
        assert "bf16x-v1" in str(err)
    else:
        raise AssertionError("wrong kind accepted")
