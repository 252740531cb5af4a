"""Failure path of the bounded device waits, without faulting or hanging the
GPU: each of the library's waits (the GEMV's mbarrier wait, the tcgen05 GEMM
roles' wait, the slab GEMM's cross-CTA counter wait, the collective GEMV's
wait for its exchange words) is run by bf16x_selftest_wait against a barrier,
flag or word that
nothing completes, with a 100 us limit.  The wait must give up, the kernel
must return, the wait-timeout bit must reach bf16x_device_status, and the
next fused GEMV on the same context must be correct."""
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200._lib import call, ptr
from bfloat16x_b200.resident import ResidentWeight
from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
from tests.gpu_util import bits_of, oracle_dict, rel_l2

pytestmark = pytest.mark.gpu
LIMIT_NS = 100_000
WAIT_TIMEOUT_BIT = 1


def _run(which, flag_value):
    # words 0..1: the u32 flag of wait 2, and the 64-bit exchange word of wait
    # 3 whose high half is the epoch it waits for (1)
    flag = torch.tensor([flag_value, flag_value], dtype=torch.int32, device="cuda")
    res = torch.full((3,), -1, dtype=torch.int32, device="cuda")
    call("bf16x_selftest_wait", which, LIMIT_NS, ptr(flag), ptr(res), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return [int(v) for v in res.cpu()], _lib.device_status()


@pytest.mark.parametrize("which", [0, 1, 2, 3])
def test_wait_runs_out_and_reports(which):
    _lib.device_status()                       # start from a clear status word
    (gave_up, aborted, waited_us), flags = _run(which, 0)
    assert gave_up == 1
    assert flags & WAIT_TIMEOUT_BIT
    assert LIMIT_NS / 1000 <= waited_us < 100_000            # returned soon after the limit
    assert aborted == (1 if which in (1, 2) else 0)          # GEMM roles also raise their abort flag
    assert _lib.device_status() == 0                         # read-and-clear
    # the context is still usable: a fused GEMV right after is correct
    w = synthetic_weight(256, 1024, seed=1)
    rw = ResidentWeight.from_packed(oracle_dict(bits_of(w)), device="cuda")
    x = synthetic_activation(2, 1024, seed=2).cuda()
    y = rw.gemv(x, out_dtype=torch.float32)
    ref = x.float() @ w.float().cuda().T
    assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < 1e-3
    assert _lib.device_status() == 0


@pytest.mark.parametrize("which", [2, 3])
def test_wait_satisfied_flag_returns_at_once(which):
    _lib.device_status()
    (gave_up, aborted, waited_us), flags = _run(which, 1)
    assert gave_up == 0 and aborted == 0 and flags == 0
    assert waited_us < LIMIT_NS / 1000


def test_selftest_rejects_long_limits():
    res = torch.zeros(3, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.Bf16xError, match="limit"):
        call("bf16x_selftest_wait", 0, 10**9, None, ptr(res), torch.cuda.current_stream().cuda_stream)
