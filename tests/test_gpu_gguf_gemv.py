"""GPU parity of the GEMV that reads GGUF BF16X blocks in place
(bf16x_gguf_gemv): against the CPU oracle's block decode + side table +
fp32 matmul (bf16x_gguf_block.py:84-95,174-188) within the 1e-3 relative-L2
gate, and bit-exact on identity probes, where every output is one decoded
weight; the side table's re-indexed records are checked entry by entry."""
import numpy as np
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200 import bf16x_gguf_block as G
from oracle import oracle
from tests.gpu_util import rel_l2

pytestmark = pytest.mark.gpu
GATE = 1e-3


def _weight(shape, seed, outlier_frac=0.005):
    """N(0, 0.02) with outliers x 2^U{4..8}: a few percent of each row needs
    the side table (more than 6 binades below its half-block's largest)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    n = int(w.size * outlier_frac)
    idx = rng.choice(w.size, n, replace=False)
    w.reshape(-1)[idx] *= np.exp2(rng.integers(4, 9, n)).astype(np.float32)
    return w


def _exact_bits(w, lossless):
    blocks = oracle.gguf_quantize_blocks(w)
    bits = oracle.gguf_dequantize_bits(blocks).reshape(w.shape)
    if lossless:
        bits = oracle.gguf_apply_ovf_bits(bits, oracle.gguf_pack_ovf(w))
    return bits


def _acts(batch, in_f, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(batch, in_f, generator=g).to(torch.bfloat16)


@pytest.mark.parametrize("lossless", [True, False])
@pytest.mark.parametrize("shape,batch", [((1000, 2048), 1), ((300, 512), 3), ((4096, 4096), 1), ((4096, 4096), 8),
                                         ((1024, 14336), 2), ((16, 256), 16), ((2000, 1024), 11), ((513, 768), 5)])
def test_gguf_gemv_vs_oracle(shape, batch, lossless):
    w = _weight(shape, 3 + batch)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=lossless, native=True)
    assert gw.gemv_in_place
    ref_bits = _exact_bits(w, lossless)
    x = _acts(batch, shape[1], batch)
    ref = oracle.matmul_bf16w(x.float().numpy(), ref_bits)
    y = gw.gemv(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, ref) < GATE
    yb = gw.gemv(x.cuda()).float().cpu().numpy()
    assert rel_l2(yb, ref) < 1e-2
    _lib.check_device_status()


def test_gguf_gemv_all_batches_and_bias():
    shape = (777, 1536)
    w = _weight(shape, 21)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=True, native=True)
    bits = _exact_bits(w, True)
    bias = torch.randn(shape[0], generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    for b in range(1, 17):
        x = _acts(b, shape[1], 100 + b)
        ref = oracle.matmul_bf16w(x.float().numpy(), bits, bias.float().numpy())
        y = gw.gemv(x.cuda(), bias=bias.cuda(), out_dtype=torch.float32).cpu().numpy()
        assert rel_l2(y, ref) < GATE, b
    _lib.check_device_status()


@pytest.mark.parametrize("lossless", [True, False])
def test_gguf_gemv_identity_probes_exact(lossless):
    """x = one-hot rows: each output is one decoded weight, exactly.  The
    zero marker's subnormal values (exponent 0) may come back as zero from
    the tensor core's fp32 result; every normal weight must match bit for bit."""
    shape = (300, 512)
    w = _weight(shape, 31, outlier_frac=0.02)
    w[5, 64:96] = 0.0                      # an all-zero block: emax floored at 7, every delta a marker
    w[7, :] = 0.0                          # an all-zero row
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=lossless, native=True)
    ref = oracle.bf16_bits_to_f32(_exact_bits(w, lossless))
    got = np.zeros_like(ref)
    for k0 in range(0, shape[1], 16):
        x = torch.zeros(16, shape[1], dtype=torch.bfloat16)
        x[torch.arange(16), torch.arange(k0, k0 + 16)] = 1.0
        got[:, k0:k0 + 16] = gw.gemv(x.cuda(), out_dtype=torch.float32).cpu().numpy().T
    normal = np.abs(ref) >= np.float32(2.0 ** -126)
    assert np.array_equal(got[normal].view(np.uint32), ref[normal].view(np.uint32))
    assert np.all(np.abs(got[~normal]) < np.float32(2.0 ** -126))
    _lib.check_device_status()


def _frag_position(entry):
    """(row, col) of a record entry: the inverse of the kernel's fragment
    slot (lane (g, t) holds block 2t + half of rows g and g + 8; step J pairs
    2J and 2J + 1; pair P = weights P and P + 16 of the block)."""
    idx = entry & 0x7FF
    half = (entry >> 11) & 1
    step = idx >> 8
    hw = idx & 1
    reg = (idx >> 1) & 3
    owner = ((idx >> 3) & 31) ^ step
    row = (owner >> 2) + 8 * (reg & 1)
    col = 32 * (2 * (owner & 3) + half) + 2 * step + (reg >> 1) + 16 * hw
    return row, col


def test_gguf_side_records_match_table():
    shape = (300, 1024)
    w = _weight(shape, 41, outlier_frac=0.01)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=True)
    item_off, recs = gw.side_records()
    off = item_off.cpu().numpy().astype(np.int64)
    rec = recs.cpu().numpy().view(np.uint32)
    ro, ec, eb = (t.cpu().numpy() for t in gw.side)
    ec = ec.view(np.uint16)
    eb = eb.view(np.uint16)
    nch = shape[1] // 256
    want = {}
    for r in range(shape[0]):
        for k in range(ro[r], ro[r + 1]):
            want[(r, int(ec[k]))] = int(eb[k])
    seen = {}
    for it in range(len(off) - 1):
        tile, c = divmod(it, nch)
        hdr = rec[off[it]]
        n_low, n_all = int(hdr & 0xFFFF), int(hdr >> 16)
        assert off[it + 1] - off[it] == (4 + n_all + 3) // 4 * 4
        assert not rec[off[it] + 1:off[it] + 4].any()
        prev = None
        for j in range(n_all):
            e = int(rec[off[it] + 4 + j])
            half = (e >> 11) & 1
            assert half == (0 if j < n_low else 1)
            r, cc = _frag_position(e)
            assert (cc >> 5) & 1 == half
            key = (half, r, cc)
            assert prev is None or key > prev          # half, then row, then column
            prev = key
            seen[(tile * 16 + r, c * 256 + cc)] = e >> 16
    assert seen == want
    _lib.check_device_status()


def test_gguf_side_table_rejects_unsorted():
    w = _weight((64, 512), 51, outlier_frac=0.02)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=True)
    ro, ec, eb = gw.side
    r = int(torch.nonzero(ro[1:] - ro[:-1] >= 2)[0, 0])
    k = int(ro[r])
    bad = ec.clone()
    bad[k], bad[k + 1] = ec[k + 1], ec[k]         # two columns of one row swapped
    gb = G.GgufWeight(gw.blocks, 64, 512, side=(ro, bad, eb))
    with pytest.raises(_lib.Bf16xError, match="ascending"):
        gb.side_records()


def test_gguf_gemv_other_in_f_uses_resident_layout():
    shape = (100, 288)                              # in_f % 256 != 0: no in-place block GEMV
    w = _weight(shape, 61)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=True, native=True)
    assert not gw.blocks_native and not gw.gemv_in_place
    x = _acts(2, shape[1], 7)
    ref = oracle.matmul_bf16w(x.float().numpy(), _exact_bits(w, True))
    y = gw.gemv(x.cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, ref) < GATE


def test_gguf_gemv_agrees_with_resident_path():
    shape = (2048, 4096)
    w = _weight(shape, 71)
    gw = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=True, native=True)
    x = _acts(4, shape[1], 9).cuda()
    a = gw.gemv(x, out_dtype=torch.float32)
    b = gw.resident().gemv(x, out_dtype=torch.float32)
    assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < 1e-5
    _lib.check_device_status()


def test_gguf_gemv_small_emax_blocks_exact():
    """Blocks no packer writes (emax below 6, where emax - delta can go
    negative and is clamped at 0 by the decode): the exact per-lane form."""
    shape = (64, 256)
    w = _weight(shape, 81)
    blocks = oracle.gguf_quantize_blocks(w).copy()          # (rows, 8, 46)
    rng = np.random.default_rng(3)
    for r, b in zip(rng.integers(0, shape[0], 40), rng.integers(0, 8, 40)):
        blocks[r, b, 0] = rng.integers(0, 6)
        blocks[r, b, 1] = rng.integers(0, 9)
    gw = G.GgufWeight.from_blocks(blocks, shape[0], shape[1], native=True)
    ref = oracle.bf16_bits_to_f32(oracle.gguf_dequantize_bits(blocks).reshape(shape))
    got = np.zeros_like(ref)
    for k0 in range(0, shape[1], 16):
        x = torch.zeros(16, shape[1], dtype=torch.bfloat16)
        x[torch.arange(16), torch.arange(k0, k0 + 16)] = 1.0
        got[:, k0:k0 + 16] = gw.gemv(x.cuda(), out_dtype=torch.float32).cpu().numpy().T
    normal = np.abs(ref) >= np.float32(2.0 ** -126)
    assert np.array_equal(got[normal].view(np.uint32), ref[normal].view(np.uint32))
    assert np.all(np.abs(got[~normal]) < np.float32(2.0 ** -126))
    _lib.check_device_status()


def test_gguf_weight_picks_gemv_path():
    w = _weight((256, 512), 91)
    lossy = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=False)
    lossless = G.GgufWeight.from_float(torch.from_numpy(w).cuda(), lossless=True)
    assert lossy.gemv_in_place and not lossless.gemv_in_place
    x = _acts(1, 512, 3)
    for gw, lo in ((lossy, False), (lossless, True)):
        ref = oracle.matmul_bf16w(x.float().numpy(), _exact_bits(w, lo))
        assert rel_l2(gw.linear(x.cuda(), out_dtype=torch.float32).cpu().numpy(), ref) < GATE
