"""GPU: the bf16x-v1 loader and packer.  The fixture written by the
reference's own packer loads into Bf16xStreamLinear layers whose resident
weights decode bit-exactly to the original bf16 and whose outputs match the
oracle matmul; this package's GPU packer writes the same files byte for
byte."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from bfloat16x_b200 import _lib
from bfloat16x_b200 import pack_to_disk as ptd
from oracle import oracle
from tests.gpu_util import bits_of, rel_l2

pytestmark = pytest.mark.gpu
GATE = 1e-3
GOLD = os.path.join(os.path.dirname(__file__), "golden")
PREFIX = os.path.join(GOLD, "disk_v1_small")
PACKED = ("up", "down", "ragged")


def _weights():
    return dict(np.load(os.path.join(GOLD, "disk_v1_small_weights.npz")))


def _model(w):
    """The fixture's module tree (names and shapes), weights from the npz."""
    m = nn.Module()
    for name in ("up", "down", "ragged", "small", "lm_head"):
        bits = w[f"{name}.weight"]
        has_b = f"{name}.bias" in w
        lin = nn.Linear(bits.shape[1], bits.shape[0], bias=has_b)
        lin.weight.data = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
        if has_b:
            lin.bias.data = torch.from_numpy(w[f"{name}.bias"].view(np.int16).copy()).view(torch.bfloat16)
        setattr(m, name, lin)
    return m


@pytest.mark.parametrize("resident", [True, False])
def test_load_reference_blob(resident):
    w = _weights()
    m = _model(w)
    n = ptd.replace_linears_from_packed(m, PREFIX, resident_fn=lambda name: resident, verbose=False)
    assert n == len(PACKED)
    assert isinstance(m.small, nn.Linear) and isinstance(m.lm_head, nn.Linear)
    for name in PACKED:
        lay = getattr(m, name)
        assert isinstance(lay, ptd.Bf16xStreamLinear) and lay.resident == resident
        if resident:
            assert np.array_equal(bits_of(lay._gpu.decode()), w[f"{name}.weight"])
        bits = w[f"{name}.weight"]
        b = w.get(f"{name}.bias")
        bias = None if b is None else oracle.bf16_bits_to_f32(b)
        for M in (1, 3, 20):
            g = torch.Generator().manual_seed(M)
            x = torch.randn(M, bits.shape[1], generator=g).to(torch.bfloat16)
            ref = oracle.matmul_bf16w(x.float().numpy(), bits, bias)
            y = lay(x.cuda()).float().cpu().numpy()
            ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
            assert rel_l2(y, ref16) < GATE, (name, M)
    _lib.check_device_status()


def test_gpu_packer_writes_reference_files(tmp_path):
    w = _weights()
    m = _model(w).cuda()
    out = str(tmp_path / "mine")
    n, total = ptd.pack_model_to_disk(m, out, verbose=False)
    assert n == len(PACKED)
    assert m.up.weight.numel() == 0 and m.lm_head.weight.numel() > 0
    with open(out + ".meta.json") as f, open(PREFIX + ".meta.json") as g:
        assert f.read() == g.read()
    with open(out + ".safetensors", "rb") as f, open(PREFIX + ".safetensors", "rb") as g:
        assert f.read() == g.read()
    # and it loads back
    m2 = _model(w)
    assert ptd.replace_linears_from_packed(m2, out, verbose=False) == len(PACKED)
    assert np.array_equal(bits_of(m2.down._gpu.decode()), w["down.weight"])
