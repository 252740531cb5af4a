"""The decoder-glue kernels (bf16x_add_rmsnorm, bf16x_rope_qkv, bf16x_silu_mul)
against the framework ops they replace in llama_e2e's CPU path, on the GPU:
bf16 outputs within one bf16 rounding step (the reductions sum in another
order), the rotary embedding and the cache write exact up to that rounding."""
import pytest
import torch
import torch.nn.functional as F

from bfloat16x_b200 import _lib
from bfloat16x_b200.llama_e2e import RMSNorm, _apply_rope, _rope_tables

pytestmark = pytest.mark.gpu


def _close(a, b, tol=1e-2):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30)) < tol


def test_add_rmsnorm_matches_framework_ops():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 5, 4096, generator=g).to(torch.bfloat16)
    d = torch.randn(3, 5, 4096, generator=g).to(torch.bfloat16)
    norm = RMSNorm(4096, 1e-5)
    norm.weight.data = (torch.rand(4096, generator=g) + 0.5).to(torch.bfloat16)
    h_ref = x + d
    y_ref = norm(h_ref)                              # CPU: framework ops
    norm.cuda()
    h, y = norm.add_forward(x.cuda(), d.cuda())
    assert torch.equal(h.cpu(), h_ref)               # the residual sum rounds the same way
    assert _close(y.cpu(), y_ref, 4e-3)
    y2 = norm(x.cuda())
    assert _close(y2.cpu(), RMSNorm(4096, 1e-5).__class__.forward(norm.cpu(), x), 4e-3)
    _lib.check_device_status()


def test_rope_qkv_matches_framework_ops():
    B, T, H, KV, D, S = 2, 3, 8, 2, 64, 40
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(B, T, (H + 2 * KV) * D, generator=g).to(torch.bfloat16)
    cos, sin = _rope_tables(D, S, 10000.0, "cpu")
    pos0 = 17
    pos = pos0 + torch.arange(T)
    q = qkv[..., :H * D].reshape(B, T, H, D)
    k = qkv[..., H * D:(H + KV) * D].reshape(B, T, KV, D)
    v = qkv[..., (H + KV) * D:].reshape(B, T, KV, D)
    q_ref, k_ref = _apply_rope(q, cos[pos], sin[pos]), _apply_rope(k, cos[pos], sin[pos])
    ck = torch.zeros(B, S, KV, D, dtype=torch.bfloat16, device="cuda")
    cv = torch.zeros_like(ck)
    qo = torch.empty(B, T, H, D, dtype=torch.bfloat16, device="cuda")
    p0 = torch.tensor(pos0, dtype=torch.long, device="cuda")
    cc, sc = cos.cuda(), sin.cuda()
    qd = qkv.cuda()
    _lib.call("bf16x_rope_qkv", qd.data_ptr(), B * T, T, H, KV, D, p0.data_ptr(), cc.data_ptr(), sc.data_ptr(),
              qo.data_ptr(), ck.data_ptr(), cv.data_ptr(), ck.stride(0), S, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _close(qo.cpu(), q_ref, 4e-3)
    assert _close(ck[:, pos0:pos0 + T].cpu(), k_ref, 4e-3)
    assert torch.equal(cv[:, pos0:pos0 + T].cpu(), v)
    assert int(ck[:, :pos0].abs().sum()) == 0 and int(ck[:, pos0 + T:].abs().sum()) == 0
    _lib.check_device_status()
    # a position past the cache is skipped and reported, nothing written
    p_bad = torch.tensor(S - 1, dtype=torch.long, device="cuda")
    ck2 = torch.zeros_like(ck)
    _lib.call("bf16x_rope_qkv", qd.data_ptr(), B * T, T, H, KV, D, p_bad.data_ptr(), cc.data_ptr(), sc.data_ptr(),
              qo.data_ptr(), ck2.data_ptr(), cv.data_ptr(), ck2.stride(0), S, torch.cuda.current_stream().cuda_stream)
    assert _lib.device_status() & 16
    assert float(ck2[:, : S - 1].abs().sum()) == 0.0


def test_silu_mul_matches_framework_ops():
    g = torch.Generator().manual_seed(2)
    gu = torch.randn(7, 2 * 1536, generator=g).to(torch.bfloat16)
    ref = F.silu(gu[:, :1536]) * gu[:, 1536:]
    out = torch.empty(7, 1536, dtype=torch.bfloat16, device="cuda")
    gd = gu.cuda()
    _lib.call("bf16x_silu_mul", gd.data_ptr(), 7, 1536, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert _close(out.cpu(), ref, 4e-3)
    _lib.check_device_status()
