"""GPU parity on the benchmarked shapes themselves, at full size.

The weights are packed on the GPU (``bf16x_quantize``, bit-exact against the
oracle in test_gpu_flat.py), the resident layout must decode back to the
input bit for bit, and the fused GEMV / GEMM outputs (fp32) must be within
the 1e-3 relative-L2 gate of the decoded-bf16 fp32-accumulate matmul.  At
these sizes the CPU oracle would take minutes, so the fp32 reference matmul
runs on the device (TF32 off) on the exact decoded weight; the oracle pins
the same computation on the small cases of test_gpu_resident.py /
test_gpu_gemm.py.  Also here: config 1 (2048x1536, seed 0) against the
output the reference itself produced (tests/golden/config1_y1.npy), and the
drop-in ``BF16XLinear`` / ``replace_with_bf16x`` (opqk_linear.py:327-440)."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from bfloat16x_b200 import _lib
from bfloat16x_b200.opqk_linear import BF16XLinear, bf16x_quantize, replace_with_bf16x
from bfloat16x_b200.resident import ResidentWeight
from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
from oracle import oracle
from tests.gpu_util import GOLD, bits_of, rel_l2

pytestmark = pytest.mark.gpu
GATE = 1e-3      # relative L2 against the decoded-bf16 fp32-accumulate matmul (fp32 outputs)
CONFIG_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]

_WEIGHTS: dict = {}


def _resident(shape, seed=0):
    """(bf16 weight on the device, its resident layout), built once per shape."""
    key = (shape, seed)
    if key not in _WEIGHTS:
        _WEIGHTS.clear()                     # keep at most one full-size weight alive
        torch.cuda.empty_cache()
        w = synthetic_weight(*shape, seed=seed, device="cuda")
        rw = ResidentWeight.from_packed(bf16x_quantize(w, device="cuda"), device="cuda")
        assert torch.equal(rw.decode().view(torch.int16), w.view(torch.int16)), "resident decode not bit-exact"
        _WEIGHTS[key] = (w, rw)
    return _WEIGHTS[key]


def _ref(x, w):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return x.float() @ w.float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _err(y, ref):
    return float((y.double() - ref.double()).norm() / ref.double().norm())


@pytest.mark.parametrize("shape", CONFIG_SHAPES)
def test_gemv_config_shape_all_batches(shape):
    w, rw = _resident(shape)
    for b in (1, 2, 4, 8):
        x = synthetic_activation(b, shape[1], seed=100 + b, device="cuda")
        y = rw.gemv(x, out_dtype=torch.float32)
        e = _err(y, _ref(x, w))
        assert e < GATE, (shape, b, e)
        # bf16 output against the rounded reference (rounding alone is ~1e-3)
        y16 = rw.gemv(x, out_dtype=torch.bfloat16)
        e16 = _err(y16.float(), _ref(x, w).to(torch.bfloat16).float())
        assert e16 < GATE, (shape, b, e16)
    assert int(rw.tile_counters.abs().sum()) == 0
    _lib.check_device_status()


@pytest.mark.parametrize("shape,M", [((14336, 4096), 512), ((14336, 4096), 2048), ((128256, 4096), 512),
                                     ((128256, 4096), 2048), ((4096, 14336), 8192), ((4096, 4096), 8192)])
def test_gemm_config_shape(shape, M):
    w, rw = _resident(shape)
    x = synthetic_activation(M, shape[1], seed=M, device="cuda")
    y = rw.gemm(x, out_dtype=torch.float32)
    ref = _ref(x, w)
    e = _err(y, ref)
    assert e < GATE, (shape, M, e)
    del y
    y16 = rw.gemm(x, out_dtype=torch.bfloat16)
    e16 = _err(y16.float(), ref.to(torch.bfloat16).float())
    assert e16 < GATE, (shape, M, e16)
    _lib.check_device_status()


def test_config1_gemv_against_reference_output():
    """Config 1: the reference's own fp32 matmul of its decoded weight."""
    yref = np.load(os.path.join(GOLD, "config1_y1.npy"))
    w = synthetic_weight(2048, 1536, seed=0)
    p = bf16x_quantize(w)
    rw = ResidentWeight.from_packed(p, device="cuda")
    assert torch.equal(rw.decode().cpu().view(torch.int16), w.view(torch.int16))
    x = synthetic_activation(1, 1536, seed=1).cuda()
    y = rw.gemv(x, out_dtype=torch.float32).cpu().numpy()
    assert y.shape == yref.shape
    assert rel_l2(y, yref) < GATE
    lin = BF16XLinear.from_packed(p)
    y2 = lin(x.float()).cpu().numpy()          # the drop-in's forward, fp32 in and out
    assert rel_l2(y2, yref) < GATE
    _lib.check_device_status()


@pytest.mark.parametrize("rows_x", [1, 7, 16, 17, 300])
def test_bf16x_linear_forward(rows_x):
    """BF16XLinear.forward (opqk_linear.py:390-404): bf16 in, bf16 out, bias
    added; <= 16 rows take the fused GEMV, more the tcgen05 GEMM."""
    out_f, in_f = 1000, 1536
    lin0 = nn.Linear(in_f, out_f, bias=True)
    with torch.no_grad():
        lin0.weight.copy_(synthetic_weight(out_f, in_f, seed=5).float())
        lin0.bias.copy_(torch.randn(out_f, generator=torch.Generator().manual_seed(2)) * 0.1)
    lin = BF16XLinear(lin0.to(torch.bfloat16))
    x = synthetic_activation(rows_x, in_f, seed=rows_x).cuda().reshape(1, rows_x, in_f)
    y = lin(x)
    assert y.shape == (1, rows_x, out_f) and y.dtype == torch.bfloat16
    wb = bits_of(lin0.weight.data)
    ref = oracle.matmul_bf16w(x.reshape(rows_x, in_f).float().cpu().numpy(), wb,
                              lin0.bias.data.float().numpy())
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    assert rel_l2(y.reshape(rows_x, out_f).float().cpu().numpy(), ref16) < GATE
    _lib.check_device_status()


def test_bf16x_linear_decode_paths():
    """decode_to_bf16 / _decode_tile / decoded_weight / clear_bf16
    (opqk_linear.py:360-388, 406-407) are bit-exact."""
    out_f, in_f = 1000, 1536
    w = synthetic_weight(out_f, in_f, seed=11)
    wb = bits_of(w)
    lin = BF16XLinear.from_packed(bf16x_quantize(w))
    full = lin.decode_to_bf16()
    assert np.array_equal(bits_of(full), wb)
    for s, e in [(0, 1000), (0, 16), (16, 48), (5, 37), (999, 1000), (640, 640), (984, 1000)]:
        t = lin._decode_tile(s, e)
        assert t.shape == (e - s, in_f)
        assert np.array_equal(bits_of(t), wb[s:e]), (s, e)
    assert np.array_equal(lin.decoded_weight().cpu().numpy(), oracle.bf16_bits_to_f32(wb))
    x = synthetic_activation(3, in_f, seed=3).cuda()
    y_dec = lin(x)                                   # F.linear on the cached decode
    lin.clear_bf16()
    y_fused = lin(x)                                 # fused kernel again
    assert rel_l2(y_dec.float().cpu().numpy(), y_fused.float().cpu().numpy()) < GATE
    _lib.check_device_status()


def test_replace_with_bf16x():
    """replace_with_bf16x (opqk_linear.py:428-440): every nn.Linear with more
    than min_el weights is replaced, smaller ones kept, the count returned."""
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(512, 256), nn.ReLU(), nn.Sequential(nn.Linear(256, 512, bias=False)),
                          nn.Linear(512, 8)).to(torch.bfloat16)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, nn.Linear):
                m.weight.copy_(synthetic_weight(*m.weight.shape, seed=m.weight.shape[0]))
    x = synthetic_activation(4, 512, seed=9)
    with torch.no_grad():
        y_ref = model.float()(x.float()).float()          # fp32 forward of the same (bf16-exact) weights
    model = model.to(torch.bfloat16)
    n = replace_with_bf16x(model, min_el=50000)
    assert n == 2
    assert isinstance(model[0], BF16XLinear) and isinstance(model[2][0], BF16XLinear)
    assert isinstance(model[3], nn.Linear)          # 4096 weights: below min_el
    model[3].cuda()
    with torch.no_grad():
        y = model(x.cuda()).float().cpu()
    assert float((y - y_ref).norm() / y_ref.norm()) < 2e-2     # bf16 activations between layers
    _lib.check_device_status()


def test_fused_gemv_new_weight_at_freed_address():
    """bf16x_fused_gemv caches the resident layout it builds from the
    reference's argument tensors; a new weight whose streams land at the
    addresses of freed ones must not get the old layout back."""
    from bfloat16x_b200.bf16x_fused import _pad1, bf16x_fused_gemv
    from tests.test_modules_host import reference_csr
    out_f, in_f = 512, 1024
    x = synthetic_activation(1, in_f, seed=3)
    addrs = []
    for seed in (1, 2, 3):
        w = synthetic_weight(out_f, in_f, seed=seed)
        p = bf16x_quantize(w)
        olk, old, oloff = reference_csr(p["delta_ovf_idx"], p["delta_ovf_val"], out_f, in_f)
        s, m, d = (_pad1(p[k].cuda()) for k in ("sign_packed", "mant_packed", "delta_packed"))
        e = p["emax"].cuda()
        olk, old, oloff = olk.cuda(), old.cuda(), oloff.cuda()
        addrs.append(s.data_ptr())
        y = bf16x_fused_gemv(x.reshape(in_f).cuda(), s, m, d, e, olk, old, oloff, out_f, in_f)
        ref = oracle.matmul_bf16w(x.float().numpy(), bits_of(w))[0]
        ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
        assert rel_l2(y.float().cpu().numpy(), ref16) < GATE, seed
        # an in-place edit of a stream is seen too (version counter): flip
        # the sign bits of row 0, which negates y[0] exactly
        if seed == 3:
            s[: in_f // 32].bitwise_not_()
            y2 = bf16x_fused_gemv(x.reshape(in_f).cuda(), s, m, d, e, olk, old, oloff, out_f, in_f)
            assert torch.equal(y2[0], -y[0]) and y[0] != 0
            assert torch.equal(y2[1:], y[1:])
        del s, m, d, e, olk, old, oloff, p, y
    _lib.check_device_status()
