"""GPU parity of the resident layout: repack + resident decode bit-exact, and
the fused decode+GEMV against the CPU oracle (fp32 output within the 1e-3
relative-L2 gate; measured errors are ~1e-6)."""
import numpy as np
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200.resident import ResidentWeight
from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
from oracle import oracle
from tests.gpu_util import bits_of, bf16_from_bits, dict_from_npz, load_flat, oracle_dict, rel_l2

pytestmark = pytest.mark.gpu
FLAT = load_flat()
CASES = list(FLAT["cases"])
GATE = 1e-3      # relative L2 against the decoded-bf16 fp32-accumulate matmul


@pytest.mark.parametrize("case", CASES)
def test_repack_decode_matches_reference(case):
    p = dict_from_npz(FLAT, case)
    rw = ResidentWeight.from_packed(p, device="cuda")
    assert np.array_equal(bits_of(rw.decode()), FLAT[f"{case}/decoded"])


@pytest.mark.parametrize("shape", [(4096, 4096), (1000, 1536), (7, 300), (40, 14336)])
def test_repack_roundtrip_and_patch_count(shape):
    w = bits_of(synthetic_weight(*shape, seed=13))
    p = oracle_dict(w)
    rw = ResidentWeight.from_packed(p, device="cuda")
    assert np.array_equal(bits_of(rw.decode()), w)
    assert rw.n_patches == expected_patches(w)
    assert rw.layout.shape[1] == (shape[1] + 255) // 256 * 384


def expected_patches(w_bits):
    """Weights whose exponent is more than 15 below the largest of their
    row-local 32-column group (columns padded to a multiple of 256)."""
    rows, in_f = w_bits.shape
    pad = (in_f + 255) // 256 * 256
    e = np.zeros((rows, pad), dtype=np.int16)
    e[:, :in_f] = (w_bits >> 7) & 0xFF
    g = e.reshape(rows, pad // 32, 32)
    d = g.max(axis=2, keepdims=True) - g
    return int((d.reshape(rows, pad)[:, :in_f] > 15).sum())


def test_repack_row_range():
    w = bits_of(synthetic_weight(300, 512, seed=17))
    p = oracle_dict(w)
    rw = ResidentWeight.from_packed(p, device="cuda", row_range=(37, 211))
    assert rw.rows == 174
    assert np.array_equal(bits_of(rw.decode()), w[37:211])


def _gemv_check(w_bits, x_bf16, rw, bias=None):
    xf = x_bf16.float().numpy()
    ref = oracle.matmul_bf16w(xf, w_bits, None if bias is None else bias.float().numpy())
    y32 = rw.gemv(x_bf16.cuda(), bias=None if bias is None else bias.cuda(), out_dtype=torch.float32)
    y16 = rw.gemv(x_bf16.cuda(), bias=None if bias is None else bias.cuda(), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    e32 = rel_l2(y32.cpu().numpy(), ref)
    assert e32 < GATE, e32
    # bf16 output: compare with the oracle rounded to bf16 (rounding alone is ~1e-3)
    ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
    e16 = rel_l2(y16.float().cpu().numpy(), ref16)
    assert e16 < GATE, e16
    return e32


@pytest.mark.parametrize("case", [c for c in CASES if f"{c}/x1" in FLAT])
@pytest.mark.parametrize("b", [1, 3, 8])
def test_gemv_matches_reference(case, b):
    yref = FLAT[f"{case}/y{b}"]
    if not np.isfinite(yref).all() or np.abs(yref).max() > 1e37:
        # sums within a factor ~30 of FLT_MAX overflow or not depending on the
        # fp32 summation order; the decoded weights themselves are checked bit
        # for bit by test_repack_decode_matches_reference
        pytest.skip("result at the fp32 overflow threshold")
    p = dict_from_npz(FLAT, case)
    rw = ResidentWeight.from_packed(p, device="cuda")
    x = bf16_from_bits(FLAT[f"{case}/x{b}"], "cuda")
    y = rw.gemv(x, out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, yref) < GATE


@pytest.mark.parametrize("shape", [(16, 256), (17, 256), (100, 512), (33, 96), (5, 300), (1000, 1536),
                                   (64, 14336), (4096, 4096)])
@pytest.mark.parametrize("b", [1, 2, 4, 5, 8, 9, 16])
def test_gemv_vs_oracle(shape, b):
    w = synthetic_weight(*shape, seed=29)
    wb = bits_of(w)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    x = synthetic_activation(b, shape[1], seed=b)
    _gemv_check(wb, x, rw)


def test_gemv_bias_and_determinism():
    w = synthetic_weight(777, 2048, seed=31)
    wb = bits_of(w)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    x = synthetic_activation(6, 2048, seed=7)
    bias = torch.randn(777).to(torch.bfloat16)
    _gemv_check(wb, x, rw, bias=bias)
    a = rw.gemv(x.cuda(), bias=bias.cuda(), out_dtype=torch.float32)
    for _ in range(5):
        b = rw.gemv(x.cuda(), bias=bias.cuda(), out_dtype=torch.float32)
        assert torch.equal(a, b)
    assert int(rw.tile_counters.abs().sum()) == 0   # split-tile counters left at zero


def test_gemv_interleaved_shapes_share_scratch():
    # weights of different shapes share the per-stream scratch; each keeps its own counters
    ws = []
    for shape in [(4096, 4096), (1000, 1536), (4096, 4096), (64, 14336)]:
        w = synthetic_weight(*shape, seed=41)
        wb = bits_of(w)
        ws.append((wb, ResidentWeight.from_packed(oracle_dict(wb), device="cuda")))
    for rep in range(2):
        for wb, rw in ws:
            for b in (1, 2, 8):
                _gemv_check(wb, synthetic_activation(b, wb.shape[1], seed=b + rep), rw)


@pytest.mark.parametrize("shape", [(14336, 4096), (4096, 14336)])
def test_gemv_config_shapes(shape):
    w = synthetic_weight(*shape, seed=0, device="cuda")
    wb = bits_of(w)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    for b in (1, 8):
        _gemv_check(wb, synthetic_activation(b, shape[1], seed=b), rw)
    _lib.check_device_status()


@pytest.mark.parametrize("shape", [(4096, 4096), (1000, 1536), (40, 14336)])
def test_bench_byte_count_matches_stored_weight(shape):
    """bench.py's host-side count of the stored weight bytes (used for the CPU
    arms' GB/s) equals what the repack actually stores."""
    import bench
    w = bits_of(synthetic_weight(*shape, seed=19))
    p = oracle_dict(w)
    rw = ResidentWeight.from_packed(p, device="cuda")
    assert bench.stored_weight_bytes(p, *shape) == rw.nbytes()


def test_repack_filtered_table():
    # tables holding only the delta > 7 entries (the reference's GPU paths
    # filter them so) repack to the same exact weights
    w = bits_of(synthetic_weight(257, 320, seed=3))
    p = oracle_dict(w)
    keep = p["delta_ovf_val"] > 7
    p["delta_ovf_idx"], p["delta_ovf_val"] = p["delta_ovf_idx"][keep], p["delta_ovf_val"][keep]
    rw = ResidentWeight.from_packed(p, device="cuda")
    assert np.array_equal(bits_of(rw.decode()), w)
    _lib.check_device_status()


# 6 rows: (4096, 1024) runs a 10-warp configuration, (8192, 4096) the one
# that keeps the CTA's whole activation block in shared memory and stages
# fewer record words (5..8 rows, in_f <= 4096, at least 8192 items)
@pytest.mark.parametrize("shape,b", [((300, 1536), 1), ((300, 1536), 8), ((300, 1536), 13), ((4096, 1024), 6),
                                     ((8192, 4096), 6)])
def test_gemv_dense_patches(shape, b):
    from tests.test_gpu_gemm import _dense_patch_weight
    wb = _dense_patch_weight(*shape, seed=9)
    rw = ResidentWeight.from_packed(oracle_dict(wb), device="cuda")
    assert rw.n_patches > wb.size // 2
    x = synthetic_activation(b, shape[1], seed=5)
    _gemv_check(wb, x, rw)
    _lib.check_device_status()
