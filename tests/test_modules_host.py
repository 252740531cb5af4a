"""Host-side logic of the drop-in modules (no GPU): the per-row overflow CSR
that the reference's Bf16xFused builds (bf16x_fused.py:165-179) converts back
to the flat overflow table the kernels read; the resident-layout cache; the
GEMV path a GGUF weight takes."""
import numpy as np
import torch

from bfloat16x_b200.bf16x_fused import csr_to_table
from tests.gpu_util import load_flat, oracle_dict
from bfloat16x_b200.synthetic import synthetic_weight
from tests.gpu_util import bits_of


def reference_csr(ovf_idx, ovf_val, out_f, in_f):
    """The reference's CSR build, restated: keep true delta > 7, sort by row
    (stable), column and delta per entry, row offsets."""
    idx = torch.as_tensor(np.asarray(ovf_idx)).to(torch.int64)
    val = torch.as_tensor(np.asarray(ovf_val)).to(torch.int64)
    keep = val > 7
    idx, val = idx[keep], val[keep]
    rows = idx // in_f
    k = idx % in_f
    order = torch.argsort(rows, stable=True)
    rows, k, val = rows[order], k[order], val[order]
    counts = torch.bincount(rows, minlength=out_f)
    offs = torch.zeros(out_f + 1, dtype=torch.int32)
    offs[1:] = counts.cumsum(0).to(torch.int32)
    return k.to(torch.int32), val.to(torch.int32), offs


def test_csr_to_table_roundtrip_golden():
    flat = load_flat()
    for case in flat["cases"]:
        w = flat[f"{case}/w"]
        out_f, in_f = w.shape
        oi, ov = flat[f"{case}/delta_ovf_idx"], flat[f"{case}/delta_ovf_val"]
        olk, old, oloff = reference_csr(oi, ov, out_f, in_f)
        ti, tv = csr_to_table(olk, old, oloff, in_f)
        keep = ov > 7
        assert np.array_equal(ti.numpy(), oi[keep].astype(np.int32))
        assert np.array_equal(tv.numpy(), ov[keep].astype(np.uint8))


def test_csr_to_table_synthetic():
    wb = bits_of(synthetic_weight(300, 1000, seed=5))
    p = oracle_dict(wb)
    olk, old, oloff = reference_csr(p["delta_ovf_idx"], p["delta_ovf_val"], 300, 1000)
    ti, tv = csr_to_table(olk, old, oloff, 1000)
    keep = p["delta_ovf_val"].numpy() > 7
    assert np.array_equal(ti.numpy(), p["delta_ovf_idx"].numpy()[keep])
    assert np.array_equal(tv.numpy(), p["delta_ovf_val"].numpy()[keep])
    assert ti.numel() > 0


def test_empty_csr():
    ti, tv = csr_to_table(torch.zeros(0, dtype=torch.int32), torch.zeros(0, dtype=torch.int32),
                          torch.zeros(5, dtype=torch.int32), 64)
    assert ti.numel() == 0 and tv.numel() == 0


def test_resident_cache_keys_on_live_objects():
    """The functional entry points' layout cache (cached_resident) reuses a
    layout only for the very stream objects it was built from, unmodified:
    another tensor at the same address (a view here; a new allocation at a
    freed address on the GPU), an in-place edit, or a dead stream rebuild."""
    import gc

    from bfloat16x_b200 import bf16x_fused as bf
    built = []

    def build():
        built.append(object())
        return built[-1]

    bf.clear_cache()
    a = torch.arange(64, dtype=torch.int32)
    b = torch.arange(16, dtype=torch.int32)
    r1 = bf.cached_resident(("t",), (a, b), build)
    assert bf.cached_resident(("t",), (a, b), build) is r1 and len(built) == 1
    view = a[:]                                   # same address, another object
    assert view.data_ptr() == a.data_ptr()
    r2 = bf.cached_resident(("t",), (view, b), build)
    assert r2 is not r1 and len(built) == 2
    b.add_(1)                                     # in-place edit: version counter moves
    r3 = bf.cached_resident(("t",), (view, b), build)
    assert r3 is not r2 and len(built) == 3
    assert bf.cached_resident(("t",), (view, b), build) is r3
    key = (("t",), view.data_ptr(), b.data_ptr())
    assert key in bf._RESIDENT_CACHE
    del view
    gc.collect()
    assert key not in bf._RESIDENT_CACHE          # evicted when its first stream died
    bf.clear_cache()


def test_gguf_weight_gemv_path_choice():
    """GgufWeight reads the blocks in place for the lossy format and takes the
    resident layout when a side table has entries, unless told otherwise;
    in_f that is not a multiple of 256 always takes the resident layout."""
    import torch

    from bfloat16x_b200.bf16x_gguf_block import GgufWeight
    blocks = torch.zeros(64 * 512 // 32 * 46, dtype=torch.uint8)
    ro = torch.zeros(65, dtype=torch.int32)
    empty = (ro, torch.zeros(0, dtype=torch.int16), torch.zeros(0, dtype=torch.int16))
    some = (ro.clone().fill_(0), torch.zeros(3, dtype=torch.int16), torch.zeros(3, dtype=torch.int16))
    assert GgufWeight(blocks, 64, 512).gemv_in_place
    assert GgufWeight(blocks, 64, 512, side=empty).gemv_in_place
    assert not GgufWeight(blocks, 64, 512, side=some).gemv_in_place
    assert GgufWeight(blocks, 64, 512, side=some, native=True).gemv_in_place
    assert not GgufWeight(blocks, 64, 512, native=False).gemv_in_place
    odd = torch.zeros(64 * 288 // 32 * 46, dtype=torch.uint8)
    assert not GgufWeight(odd, 64, 288, native=True).gemv_in_place
