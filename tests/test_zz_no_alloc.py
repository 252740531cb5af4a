"""bf16x_gemv_noalloc (fixed device scratch, nothing allocated) against
bf16x_gemv with caller-owned counters and scratch, both through the C ABI.

Named to be collected last: it must pass both alone in a fresh process and
after every other test has used the library.  Each case makes two no-alloc
calls in a row, so the second one sees the fixed scratch exactly as the first
left it."""
import numpy as np
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200._lib import BF16X_DTYPE_BF16, BF16X_DTYPE_F32, call, ptr
from bfloat16x_b200.resident import ResidentWeight
from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
from tests.gpu_util import bits_of, oracle_dict, rel_l2

pytestmark = pytest.mark.gpu
GATE = 1e-3      # the GEMV tests' relative-L2 tolerance


def _weight(rows, in_f, seed):
    w = bits_of(synthetic_weight(rows, in_f, seed=seed))
    return ResidentWeight.from_packed(oracle_dict(w), device="cuda")


def _x(rw, batch, seed):
    x = synthetic_activation(batch, rw.in_f, seed=seed).to(torch.bfloat16)
    xp = torch.zeros((batch, rw.in_pad), dtype=torch.bfloat16, device="cuda")
    xp[:, : rw.in_f] = x.cuda()
    return xp


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _gemv_owned(rw, xp, bias, y):
    counters = torch.zeros((rw.rows + 15) // 16, dtype=torch.int32, device="cuda")
    need = int(_lib.lib().bf16x_gemv_scratch_bytes(rw.rows, rw.in_f))
    scratch = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    ydt = BF16X_DTYPE_F32 if y.dtype == torch.float32 else BF16X_DTYPE_BF16
    call("bf16x_gemv", ptr(rw.layout), ptr(rw.ptile_off), ptr(rw.precs), rw.rows, rw.in_f,
         ptr(xp), xp.shape[0], xp.stride(0), ptr(bias), ptr(y), ydt, y.stride(0), ptr(counters),
         ptr(scratch), scratch.numel(), _stream())


def _gemv_noalloc(rw, xp, bias, y):
    ydt = BF16X_DTYPE_F32 if y.dtype == torch.float32 else BF16X_DTYPE_BF16
    call("bf16x_gemv_noalloc", ptr(rw.layout), ptr(rw.ptile_off), ptr(rw.precs), rw.rows, rw.in_f,
         ptr(xp), xp.shape[0], xp.stride(0), ptr(bias), ptr(y), ydt, y.stride(0), _stream())


@pytest.mark.parametrize("shape,batch,dtype", [
    ((4096, 4096), 1, torch.float32),
    ((1000, 1536), 3, torch.float32),
    ((64, 14336), 8, torch.bfloat16),
    ((14336, 4096), 2, torch.float32),
    ((33, 96), 5, torch.bfloat16),
    # 6 rows on 8192 x 4096: the 12-warp configuration that keeps the CTA's
    # whole activation block in shared memory (most warps, most partial sums)
    ((8192, 4096), 6, torch.float32),
])
def test_noalloc_matches_gemv_twice(shape, batch, dtype):
    rw = _weight(*shape, seed=41)
    xp = _x(rw, batch, seed=43)
    bias = (torch.randn(rw.rows, generator=torch.Generator().manual_seed(47)) * 0.1).to(torch.bfloat16).cuda()
    y_ref = torch.empty((batch, rw.rows), dtype=dtype, device="cuda")
    _gemv_owned(rw, xp, bias, y_ref)
    outs = []
    for _ in range(2):
        y = torch.full((batch, rw.rows), float("nan"), dtype=dtype, device="cuda")
        _gemv_noalloc(rw, xp, bias, y)
        outs.append(y)
    torch.cuda.synchronize()
    _lib.check_device_status()
    ref = y_ref.float().cpu().numpy()
    for y in outs:
        got = y.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, ref) < GATE
    # the same kernel and the same deterministic reduction order
    assert torch.equal(outs[0], y_ref) and torch.equal(outs[1], y_ref)


def test_noalloc_rejects_oversize():
    limit = int(_lib.lib().bf16x_gemv_noalloc_max_rows())
    assert limit == 524288
    rw = _weight(64, 512, seed=53)
    xp = _x(rw, 1, seed=59)
    y = torch.empty((1, limit + 16), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.Bf16xError, match="fixed scratch limit"):
        # the size check comes before any pointer is used
        call("bf16x_gemv_noalloc", ptr(rw.layout), ptr(rw.ptile_off), ptr(rw.precs), limit + 16, rw.in_f,
             ptr(xp), 1, xp.stride(0), None, ptr(y), BF16X_DTYPE_F32, y.stride(0), _stream())


def test_noalloc_rejects_batch_above_8():
    # 9..16 activation rows need twice the partial sums of the fixed scratch;
    # bf16x_gemv takes them, the no-alloc entry point refuses them up front
    rw = _weight(64, 512, seed=61)
    xp = _x(rw, 9, seed=67)
    y = torch.empty((9, rw.rows), dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.Bf16xError, match="batch must be 1..8"):
        _gemv_noalloc(rw, xp, None, y)
    y_ref = torch.empty_like(y)
    _gemv_owned(rw, xp, None, y_ref)
    torch.cuda.synchronize()
    assert np.isfinite(y_ref.cpu().numpy()).all()
