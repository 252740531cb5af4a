"""GPU parity of the tcgen05 decode+GEMM: identity probes (bit-exact: each
output equals one decoded weight), then random activations against the CPU
oracle within the 1e-3 relative-L2 gate, ragged shapes included."""
import numpy as np
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200.resident import ResidentWeight
from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
from oracle import oracle
from tests.gpu_util import bits_of, oracle_dict, rel_l2

pytestmark = pytest.mark.gpu
GATE = 1e-3


@pytest.mark.parametrize("shape,M", [((128, 256), 64), ((256, 512), 256), ((300, 1536), 130), ((200, 320), 300)])
def test_gemm_identity_probe(shape, M):
    # x = one-hot rows: y[m, n] = W[n, m] exactly (fp32 of the bf16 weight)
    rows, in_f = shape
    w = synthetic_weight(rows, in_f, seed=3)
    wb = bits_of(w)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    M = min(M, in_f)
    x = torch.zeros(M, in_f, dtype=torch.bfloat16)
    x[torch.arange(M), torch.arange(M)] = 1.0
    y = rw.gemm(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    expect = oracle.bf16_bits_to_f32(wb)[:, :M].T
    assert np.array_equal(y.view(np.uint32), np.ascontiguousarray(expect).view(np.uint32))
    _lib.check_device_status()


@pytest.mark.parametrize("shape", [(128, 256), (1000, 1536), (333, 4099), (4096, 4096), (200, 14336)])
@pytest.mark.parametrize("M", [9, 64, 200, 512])
def test_gemm_vs_oracle(shape, M):
    w = synthetic_weight(*shape, seed=5)
    wb = bits_of(w)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    x = synthetic_activation(M, shape[1], seed=M)
    ref = oracle.matmul_bf16w(x.float().numpy(), wb)
    y32 = rw.gemm(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y32, ref) < GATE
    y16 = rw.gemm(x.cuda(), out_dtype=torch.bfloat16).float().cpu().numpy()
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    assert rel_l2(y16, ref16) < GATE


def test_gemm_bias_and_dispatch():
    w = synthetic_weight(640, 2048, seed=9)
    wb = bits_of(w)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    bias = torch.randn(640).to(torch.bfloat16)
    for M in (3, 8, 9, 300):
        x = synthetic_activation(M, 2048, seed=M)
        ref = oracle.matmul_bf16w(x.float().numpy(), wb, bias.float().numpy())
        y = rw.linear(x.cuda(), bias=bias.cuda(), out_dtype=torch.float32).cpu().numpy()
        assert rel_l2(y, ref) < GATE, M
    _lib.check_device_status()


def test_gemm_large_m_deterministic():
    w = synthetic_weight(4096, 4096, seed=1, device="cuda")
    rw = ResidentWeight.from_packed(oracle_dict(bits_of(w)), device="cuda")
    x = synthetic_activation(2048, 4096, seed=2, device="cuda")
    a = rw.gemm(x, out_dtype=torch.float32)
    b = rw.gemm(x, out_dtype=torch.float32)
    assert torch.equal(a, b)
    ref = x.float() @ w.float().T
    assert float((a - ref).norm() / ref.norm()) < GATE


def _dense_patch_weight(rows, in_f, seed):
    # magnitudes spread over 2^-40..2^0: most weights sit more than 15 binades
    # below their 32-column maximum, so records overflow every staging limit
    g = torch.Generator().manual_seed(seed)
    e = torch.randint(-40, 1, (rows, in_f), generator=g).float()
    m = 1.0 + torch.rand(rows, in_f, generator=g)
    s = torch.where(torch.rand(rows, in_f, generator=g) < 0.5, -1.0, 1.0)
    return bits_of((s * m * torch.exp2(e)).to(torch.bfloat16))


@pytest.mark.parametrize("shape,M", [((256, 512), 200), ((300, 1536), 64)])
def test_gemm_dense_patches(shape, M):
    wb = _dense_patch_weight(*shape, seed=7)
    p = oracle_dict(wb)
    rw = ResidentWeight.from_packed(p, device="cuda")
    assert rw.n_patches > wb.size // 2
    assert np.array_equal(bits_of(rw.decode()), wb)
    x = synthetic_activation(M, shape[1], seed=3)
    y = rw.gemm(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    ref = oracle.matmul_bf16w(x.float().numpy(), wb)
    assert rel_l2(y, ref) < GATE
    _lib.check_device_status()


# Shapes with at least 148 tiles of 128 rows x 256 tokens run the CTA-pair
# kernel (cluster of 2, tiles of 256 rows x 256 tokens).
@pytest.mark.parametrize("rows,in_f,M", [(8192, 1024, 768), (8192, 1024, 1024), (8192, 2048, 2048)])
def test_gemm_pair_identity_probe(rows, in_f, M):
    wb = bits_of(synthetic_weight(rows, in_f, seed=21))
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    x = torch.eye(M, in_f, dtype=torch.bfloat16)
    y = rw.gemm(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    expect = oracle.bf16_bits_to_f32(wb)[:, :M].T
    assert np.array_equal(y.view(np.uint32), np.ascontiguousarray(expect).view(np.uint32))
    _lib.check_device_status()


# 4196 rows: the last pair tile has 100 rows (all in the leader CTA); 2597
# tokens: the last token tile is ragged in both CTAs' halves; 8100 rows at
# 700 tokens: ragged in rows and in tokens with 96 tiles
@pytest.mark.parametrize("rows,M", [(4196, 2597), (8100, 700)])
@pytest.mark.parametrize("dense", [False, True])
def test_gemm_pair_ragged_vs_oracle(rows, M, dense):
    in_f = 1024
    wb = _dense_patch_weight(rows, in_f, seed=5) if dense else bits_of(synthetic_weight(rows, in_f, seed=23))
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    bias = (torch.randn(rows, generator=torch.Generator().manual_seed(1)) * 0.1).to(torch.bfloat16)
    x = synthetic_activation(M, in_f, seed=29)
    ref = oracle.matmul_bf16w(x.float().numpy(), wb, bias.float().numpy())
    y = rw.gemm(x.cuda(), bias=bias.cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, ref) < GATE
    y16 = rw.gemm(x.cuda(), bias=bias.cuda(), out_dtype=torch.bfloat16).float().cpu().numpy()
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    assert rel_l2(y16, ref16) < GATE
    _lib.check_device_status()


# 257..512 tokens on shapes that fill the GPU with pair tiles run 512-token
# pair tiles (each CTA stages two 128-token blocks; two N=256 MMAs per
# k-block): the identity probe checks every token's column in all four
# blocks, the ragged case a tile with 300 of 512 tokens and partial rows.
@pytest.mark.parametrize("rows,in_f,M", [(9600, 1024, 512), (9728, 512, 384)])
def test_gemm_pair512_identity_probe(rows, in_f, M):
    wb = bits_of(synthetic_weight(rows, in_f, seed=31))
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    x = torch.eye(M, in_f, dtype=torch.bfloat16)
    y = rw.gemm(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    expect = oracle.bf16_bits_to_f32(wb)[:, :M].T
    assert np.array_equal(y.view(np.uint32), np.ascontiguousarray(expect).view(np.uint32))
    _lib.check_device_status()


@pytest.mark.parametrize("dense", [False, True])
def test_gemm_pair512_ragged_vs_oracle(dense):
    rows, in_f, M = 9700, 1024, 300
    wb = _dense_patch_weight(rows, in_f, seed=7) if dense else bits_of(synthetic_weight(rows, in_f, seed=37))
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    bias = (torch.randn(rows, generator=torch.Generator().manual_seed(2)) * 0.1).to(torch.bfloat16)
    x = synthetic_activation(M, in_f, seed=41)
    ref = oracle.matmul_bf16w(x.float().numpy(), wb, bias.float().numpy())
    y = rw.gemm(x.cuda(), bias=bias.cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, ref) < GATE
    _lib.check_device_status()


# Slab path (bf16x_gemm_ws with a workspace, at least 4 token tiles per
# 256-row slab): 16 slabs through a ring of 12 slots, and K = 14336 (56
# chunks) through a 42-chunk window, so slots are reused and windows wrap.
# x is a permuted one-hot matrix, so every output is one decoded weight and
# the columns checked span every chunk.
def test_gemm_slab_permuted_identity():
    rows, in_f, M = 4096, 14336, 2048
    assert _lib.lib().bf16x_gemm_workspace_bytes(rows, in_f, M) > 0
    wb = bits_of(synthetic_weight(rows, in_f, seed=31))
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    cols = (np.arange(M) * 5 + 3) % in_f
    x = torch.zeros(M, in_f, dtype=torch.bfloat16)
    x[torch.arange(M), torch.from_numpy(cols)] = 1.0
    y = rw.gemm(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    expect = oracle.bf16_bits_to_f32(wb)[:, cols].T
    assert np.array_equal(y.view(np.uint32), np.ascontiguousarray(expect).view(np.uint32))
    _lib.check_device_status()


# Ragged everywhere on the slab path: 5000 rows (the last slab holds 136
# rows in 9 tiles), in_f 11000 (ragged last chunk, window wraps), 1500
# tokens; against the fp32 matmul of the decoded weight (bit-exact decode is
# pinned by the decode tests), twice for determinism.
def test_gemm_slab_ragged_vs_torch():
    rows, in_f, M = 5000, 11000, 1500
    assert _lib.lib().bf16x_gemm_workspace_bytes(rows, in_f, M) > 0
    w = synthetic_weight(rows, in_f, seed=37, device="cuda")
    rw = ResidentWeight.from_packed(oracle_dict(bits_of(w)), device="cuda")
    assert torch.equal(rw.decode(), w)
    x = synthetic_activation(M, in_f, seed=41, device="cuda")
    bias = (torch.randn(rows, generator=torch.Generator().manual_seed(2)) * 0.1).to(torch.bfloat16).cuda()
    ref = x.float() @ w.float().T + bias.float()
    y = rw.gemm(x, bias=bias, out_dtype=torch.float32)
    assert float((y - ref).norm() / ref.norm()) < GATE
    assert torch.equal(y, rw.gemm(x, bias=bias, out_dtype=torch.float32))
    y16 = rw.gemm(x, bias=bias, out_dtype=torch.bfloat16).float()
    assert float((y16 - ref.to(torch.bfloat16).float()).norm() / ref.norm()) < GATE
    _lib.check_device_status()


# Slab path with 512-token tiles (two N=256 MMAs per staged k-block, the
# accumulator handed back in halves; chosen for K >= 8192): 4500 rows (the
# last slab holds 148 rows), in_f 8300 (ragged last chunk), 4200 tokens (the
# last tile holds 104, all in the first half of the leader CTA).
def test_gemm_slab_wide_ragged_vs_torch():
    rows, in_f, M = 4500, 8300, 4200
    assert _lib.lib().bf16x_gemm_workspace_bytes(rows, in_f, M) > 0
    w = synthetic_weight(rows, in_f, seed=43, device="cuda")
    rw = ResidentWeight.from_packed(oracle_dict(bits_of(w)), device="cuda")
    x = synthetic_activation(M, in_f, seed=47, device="cuda")
    bias = (torch.randn(rows, generator=torch.Generator().manual_seed(3)) * 0.1).to(torch.bfloat16).cuda()
    ref = x.float() @ w.float().T + bias.float()
    y = rw.gemm(x, bias=bias, out_dtype=torch.float32)
    assert float((y - ref).norm() / ref.norm()) < GATE
    assert torch.equal(y, rw.gemm(x, bias=bias, out_dtype=torch.float32))
    _lib.check_device_status()
