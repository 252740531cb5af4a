"""GPU parity of the drop-in modules mirroring bf16x_fused.py and
bf16x_gemm_fused.py: the stand-alone fused GEMV/GEMM functions on the
reference's own argument forms (padded streams, per-row overflow CSR), the
three Bf16xFused modes, Bf16xGemmLinear resident and streamed from pinned
host memory, and the deploy walkers on a small model.  Outputs are checked
against the CPU oracle within the 1e-3 relative-L2 gate."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from bfloat16x_b200 import _lib
from bfloat16x_b200.bf16x_fused import Bf16xFused, _pad1, bf16x_fused_gemv, deploy_bf16x_fused
from bfloat16x_b200.bf16x_gemm_fused import Bf16xGemmLinear, bf16x_fused_gemm, deploy_bf16x_gemm
from bfloat16x_b200.opqk_linear import bf16x_quantize, packed_nbytes
from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
from oracle import oracle
from tests.gpu_util import bits_of, oracle_dict, rel_l2
from tests.test_modules_host import reference_csr

pytestmark = pytest.mark.gpu
GATE = 1e-3


def _weight(shape, seed):
    wb = bits_of(synthetic_weight(*shape, seed=seed))
    return wb, oracle_dict(wb)


@pytest.mark.parametrize("shape", [(4096, 4096), (1000, 1536), (33, 96), (128, 300)])
def test_fused_gemv_reference_arguments(shape):
    wb, p = _weight(shape, 61)
    out_f, in_f = shape
    olk, old, oloff = reference_csr(p["delta_ovf_idx"], p["delta_ovf_val"], out_f, in_f)
    dev = "cuda"
    s, m, d = (_pad1(p[k].cuda()) for k in ("sign_packed", "mant_packed", "delta_packed"))
    e = p["emax"].cuda()
    x = synthetic_activation(1, in_f, seed=7)
    ref = oracle.matmul_bf16w(x.float().numpy(), wb)[0]
    for _ in range(2):                      # second call reuses the cached resident layout
        y = bf16x_fused_gemv(x.reshape(in_f).to(dev), s, m, d, e, olk.to(dev), old.to(dev), oloff.to(dev),
                             out_f, in_f)
        assert y.dtype == torch.bfloat16 and y.shape == (out_f,)
        ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
        assert rel_l2(y.float().cpu().numpy(), ref16) < GATE
    _lib.check_device_status()


@pytest.mark.parametrize("rows_x", [1, 5, 64])
def test_bf16x_fused_modes_agree(rows_x):
    wb, p = _weight((512, 768), 67)
    bias = (torch.randn(512, generator=torch.Generator().manual_seed(3)) * 0.1).to(torch.bfloat16)
    lay = Bf16xFused(p, bias=bias)
    x = synthetic_activation(rows_x, 768, seed=71).cuda()
    ref = oracle.matmul_bf16w(x.float().cpu().numpy(), wb, bias.float().numpy())
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    outs = {}
    for mode in ("fused", "opt", "repo"):
        lay.mode = mode
        y = lay(x)
        assert y.shape == (rows_x, 512) and y.dtype == torch.bfloat16
        outs[mode] = y.float().cpu().numpy()
        assert rel_l2(outs[mode], ref16) < GATE, mode
    _lib.check_device_status()


@pytest.mark.parametrize("exact", [False, True])
def test_fused_gemm_reference_arguments(exact):
    wb, p = _weight((640, 1024), 73)
    M = 300
    x = synthetic_activation(M, 1024, seed=79).cuda()
    s, m, d = (_pad1(p[k].cuda()) for k in ("sign_packed", "mant_packed", "delta_packed"))
    e = p["emax"].cuda()
    if exact:
        y = bf16x_fused_gemm(x, s, m, d, e, 640, 1024, ovf_idx=p["delta_ovf_idx"], ovf_val=p["delta_ovf_val"])
        w_used = wb
    else:
        # the reference GEMM ignores the overflow table: saturated decode
        y = bf16x_fused_gemm(x, s, m, d, e, 640, 1024)
        sat = dict(p)
        sat["delta_ovf_idx"] = np.zeros(0, np.int32)
        sat["delta_ovf_val"] = np.zeros(0, np.uint8)
        w_used = oracle.decode({k: (v.numpy() if torch.is_tensor(v) else v) for k, v in sat.items()})
    assert y.dtype == x.dtype and y.shape == (M, 640)
    ref = oracle.matmul_bf16w(x.float().cpu().numpy(), w_used)
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    assert rel_l2(y.float().cpu().numpy(), ref16) < GATE
    _lib.check_device_status()


@pytest.mark.parametrize("resident", [True, False])
@pytest.mark.parametrize("M", [3, 200])
def test_gemm_linear_resident_and_streamed(resident, M):
    wb, p = _weight((384, 2048), 83)
    bias = (torch.randn(384, generator=torch.Generator().manual_seed(5)) * 0.1).to(torch.bfloat16)
    lay = Bf16xGemmLinear(p, bias=bias, resident=resident)
    x = synthetic_activation(M, 2048, seed=89).cuda()
    ref = oracle.matmul_bf16w(x.float().cpu().numpy(), wb, bias.float().numpy())
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    for _ in range(2):
        y = lay(x)
        assert rel_l2(y.float().cpu().numpy(), ref16) < GATE
    _lib.check_device_status()


def _toy_model(seed):
    torch.manual_seed(seed)
    m = nn.Sequential()
    m.add_module("up", nn.Linear(256, 512, bias=True))
    m.add_module("act", nn.SiLU())
    m.add_module("down", nn.Linear(512, 256, bias=False))
    m.add_module("lm_head", nn.Linear(256, 300, bias=False))
    for mod in m.modules():
        if isinstance(mod, nn.Linear):
            mod.weight.data.normal_(0, 0.02)
    return m.to(torch.bfloat16).cuda()


def _ref_forward(m, x):
    h = x.float() @ m.up.weight.float().T + m.up.bias.float()
    h = torch.nn.functional.silu(h).to(torch.bfloat16).float()
    h = (h @ m.down.weight.float().T).to(torch.bfloat16).float()
    return h @ m.lm_head.weight.float().T


@pytest.mark.parametrize("which", ["fused", "gemm"])
@torch.no_grad()
def test_deploy_walkers(which):
    m = _toy_model(11)
    x = synthetic_activation(4, 256, seed=97).cuda()
    ref = _ref_forward(m, x).cpu().numpy()
    expect_total = sum(packed_nbytes(bf16x_quantize(mod.weight.data.to(torch.bfloat16)))
                       for name, mod in m.named_modules() if isinstance(mod, nn.Linear) and name != "lm_head")
    if which == "fused":
        total, n_el = deploy_bf16x_fused(m, verbose=False)
        assert isinstance(m.up, Bf16xFused) and isinstance(m.lm_head, nn.Linear)
    else:
        total, n_el = deploy_bf16x_gemm(m, verbose=False, resident_fn=lambda name: name != "down")
        assert isinstance(m.down, Bf16xGemmLinear) and not m.down.resident
    assert total == expect_total and n_el == 256 * 512 * 2
    y = m(x).float().cpu().numpy()
    assert rel_l2(y, ref) < 1e-2      # two bf16 roundings of the hidden states
    _lib.check_device_status()
