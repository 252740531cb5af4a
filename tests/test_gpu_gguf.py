"""GPU parity of the GGUF BF16X block format (bf16x_gguf_block.py mirror):
blocks, dequantized values, the lossless side table and its application are
bit-exact against the golden vectors made by the reference and against the
CPU oracle at larger sizes; the GGUF-variant weight feeds the fused GEMV and
GEMM kernels, checked against the oracle within the 1e-3 relative-L2 gate."""
import numpy as np
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200 import bf16x_gguf_block as G
from oracle import oracle
from tests.gpu_util import GOLD, rel_l2

pytestmark = pytest.mark.gpu
GGUF = np.load(f"{GOLD}/gguf_small.npz")
GATE = 1e-3


@pytest.mark.parametrize("case", [c for c in GGUF["cases"] if c != "g_special"])
def test_gguf_golden(case):
    x = GGUF[f"{case}/x"]
    blocks = G.quantize_blocks(x)
    assert np.array_equal(blocks, GGUF[f"{case}/blocks"])
    deq = G.dequantize_blocks(blocks)
    assert np.array_equal(deq.view(np.uint32), GGUF[f"{case}/deq"].reshape(x.shape).view(np.uint32))
    blob = G.pack_ovf(x)
    assert blob == GGUF[f"{case}/ovf"].tobytes()
    lossless = G.dequantize_lossless(blocks, blob)
    assert np.array_equal(lossless.view(np.uint32), GGUF[f"{case}/lossless"].view(np.uint32))
    _lib.check_device_status()


def test_gguf_special_values():
    x = GGUF["g_special/x"]
    blocks = G.quantize_blocks(x)
    assert np.array_equal(blocks, GGUF["g_special/blocks"])
    deq = G.dequantize_blocks(blocks)
    assert np.array_equal(deq.view(np.uint32), GGUF["g_special/deq"].reshape(x.shape).view(np.uint32))
    assert G.pack_ovf(x, bf16_exact=True) == GGUF["g_special/ovf"].tobytes()


def _heavy(shape, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(shape) * 0.13).astype(np.float32)
    idx = rng.choice(w.size, w.size // 200, replace=False)
    w.reshape(-1)[idx] *= rng.standard_normal(len(idx)) * 8
    return w


@pytest.mark.parametrize("shape", [(1024, 2048), (300, 576), (129, 4096), (3, 65536)])
def test_gguf_vs_oracle(shape):
    w = _heavy(shape, 7)
    blocks = G.quantize_blocks(w)
    assert np.array_equal(blocks.reshape(-1), oracle.gguf_quantize_blocks(w).reshape(-1))
    bits = G.dequantize_blocks(torch.from_numpy(blocks).cuda(), out_dtype=torch.bfloat16)
    assert np.array_equal(bits.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1),
                          oracle.gguf_dequantize_bits(blocks).reshape(-1))
    assert G.pack_ovf(w) == oracle.gguf_pack_ovf(w)
    lossless = G.dequantize_lossless(blocks, G.pack_ovf(w)).reshape(shape)
    assert np.array_equal(oracle.f32_to_bf16_bits(lossless), oracle.f32_to_bf16_bits(w))
    n, tot = G.ovf_stats(w)
    mask = G.ovf_overflow_mask(w)
    assert mask.sum() == n and tot == w.size


def test_gguf_torch_bf16_input_matches_float_path():
    w = _heavy((256, 512), 11)
    wb = torch.from_numpy(w).to(torch.bfloat16).cuda()
    b_t = G.quantize_blocks(wb)
    assert b_t.is_cuda
    exact_f32 = wb.float().cpu().numpy()
    assert np.array_equal(b_t.cpu().numpy(), G.quantize_blocks(exact_f32))
    assert G.pack_ovf(wb) == G.pack_ovf(exact_f32, bf16_exact=True)


def test_gguf_empty_side_table():
    w = np.zeros((4, 64), np.float32)
    blob = G.pack_ovf(w)
    rows, ro, c, b = G.unpack_ovf(blob)
    assert rows == 4 and ro.tolist() == [0] * 5 and c.size == 0
    assert np.array_equal(G.dequantize_lossless(G.quantize_blocks(w), blob), w.reshape(-1))


@pytest.mark.parametrize("lossless", [True, False])
def test_gguf_weight_fused_matmul(lossless):
    shape = (1000, 2048)
    w = _heavy(shape, 13)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=lossless)
    deq = gw.dequantize()
    deq_bits = deq.view(torch.int16).cpu().numpy().view(np.uint16)
    if lossless:
        assert np.array_equal(deq_bits, oracle.f32_to_bf16_bits(w))
    else:
        assert np.array_equal(deq_bits.reshape(-1), oracle.gguf_dequantize_bits(G.quantize_blocks(w)).reshape(-1))
    rw = gw.resident()
    assert np.array_equal(rw.decode().view(torch.int16).cpu().numpy().view(np.uint16), deq_bits)
    for M in (1, 5, 300):
        x = torch.randn(M, shape[1], generator=torch.Generator().manual_seed(M)).to(torch.bfloat16)
        y = gw.linear(x.cuda(), out_dtype=torch.float32).cpu().numpy()
        ref = oracle.matmul_bf16w(x.float().numpy(), deq_bits)
        assert rel_l2(y, ref) < GATE, M
    _lib.check_device_status()
