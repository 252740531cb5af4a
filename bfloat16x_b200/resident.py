"""Device-resident BF16X weights in the kernel layout.

``ResidentWeight`` is what the fused Linear modules hold: the weight rows in
the resident layout (chunks of 256 columns, 384 bytes each: sign|mant bytes
and pair-aligned 4-bit deltas -- 12 bits per weight) plus a record per
(16-row tile, 256-column chunk) holding the emax of every 32-column group of
its rows (1/4 bit per weight) and the rare weights whose exponent is more
than 15 below their group's largest.  It is built once from a
bf16x_quantize dict by the ``bf16x_repack_count`` / ``bf16x_repack`` kernels
(the counterpart of the reference modules' device preparation,
bf16x_fused.py:154-192 and bf16x_gemm_fused.py:163-184) and can hold a row
range only (tensor-parallel shards by output rows).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import BF16X_DTYPE_BF16, BF16X_DTYPE_F32, CHUNK_BYTES, CHUNK_ELEMS, REC_HDR_WORD, TILE_ROWS, call, ptr

_FLAT = ("sign_packed", "mant_packed", "delta_packed", "emax", "delta_ovf_idx", "delta_ovf_val")

GEMV_MAX_BATCH = 16


def _as_dev(t: torch.Tensor, dtype, dev) -> torch.Tensor:
    return t.to(device=dev, dtype=dtype, non_blocking=True).contiguous()


def flat_on_device(p: dict, dev) -> dict:
    """The dict's streams as contiguous device tensors of the C-ABI dtypes."""
    out = {
        "sign_packed": _as_dev(p["sign_packed"], torch.int32, dev),
        "mant_packed": _as_dev(p["mant_packed"], torch.int32, dev),
        "delta_packed": _as_dev(p["delta_packed"], torch.int32, dev),
        "emax": _as_dev(p["emax"], torch.uint8, dev),
        "delta_ovf_idx": _as_dev(p["delta_ovf_idx"], torch.int32, dev),
        "delta_ovf_val": _as_dev(p["delta_ovf_val"], torch.uint8, dev),
    }
    return out


def flat_args(f: dict):
    """Positional stream arguments of the flat-stream C entry points."""
    n_ovf = f["delta_ovf_idx"].numel()
    return (ptr(f["sign_packed"]), f["sign_packed"].numel(), ptr(f["mant_packed"]), f["mant_packed"].numel(),
            ptr(f["delta_packed"]), f["delta_packed"].numel(), ptr(f["emax"]), f["emax"].numel(),
            ptr(f["delta_ovf_idx"]) if n_ovf else None, ptr(f["delta_ovf_val"]) if n_ovf else None, n_ovf)


_SCRATCH: dict = {}
_YDT = {torch.bfloat16: BF16X_DTYPE_BF16, torch.float32: BF16X_DTYPE_F32}


def gemv_scratch(device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
    """GEMV partial-sum scratch for (device, stream: default the current one),
    grown on demand.  Its contents never need initialising."""
    if stream is None:
        stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    ws = _SCRATCH.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _SCRATCH[key] = ws
    return ws


_GEMM_WS: dict = {}


def gemm_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Slab-ring workspace of the GEMM for (device, current stream), grown on
    demand; its contents never need initialising."""
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    ws = _GEMM_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _GEMM_WS[key] = ws
    return ws


_ALL_COUNTERS: list = []


def reset_workspaces() -> None:
    """Re-zero the tile counters of every weight (after a kernel reported an
    error, a counter may have been left non-zero)."""
    for ref in list(_ALL_COUNTERS):
        t = ref()
        if t is not None:
            t.zero_()


class ResidentWeight:
    """Rows [row0, row1) of a BF16X weight in the resident kernel layout."""

    def __init__(self, layout: torch.Tensor, ptile_off: torch.Tensor, precs: torch.Tensor,
                 rows: int, in_f: int, out_f: int | None = None, row0: int = 0):
        self.layout = layout
        self.ptile_off = ptile_off
        self.precs = precs
        self.rows = int(rows)
        self.in_f = int(in_f)
        self.out_f = int(out_f if out_f is not None else rows)
        self.row0 = int(row0)
        self._n_patches = None
        self._scratch_need = None
        self._wptrs = None
        # one zeroed counter per 16-row tile, reset by the kernel after use
        self.tile_counters = torch.zeros((self.rows + TILE_ROWS - 1) // TILE_ROWS + 1, dtype=torch.int32,
                                         device=layout.device)
        import weakref
        _ALL_COUNTERS.append(weakref.ref(self.tile_counters))

    # ------------------------------------------------------------------ build
    @classmethod
    @torch.no_grad()
    def from_packed(cls, p: dict, device=None, row_range: tuple | None = None) -> "ResidentWeight":
        out_f, in_f = int(p["out_f"]), int(p["in_f"])
        if int(p.get("sub", 16)) != 16:
            raise ValueError("only sub=16 dicts are supported")
        if device is None:
            device = p["sign_packed"].device if p["sign_packed"].is_cuda else torch.device(
                "cuda", torch.cuda.current_device())
        dev = torch.device(device)
        if dev.type != "cuda":
            raise _lib.Bf16xError("ResidentWeight lives on a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        r0, r1 = (0, out_f) if row_range is None else (int(row_range[0]), int(row_range[1]))
        rows = r1 - r0
        f = flat_on_device(p, dev)
        row_bytes = int(_lib.lib().bf16x_resident_row_bytes(in_f))
        nch = (in_f + CHUNK_ELEMS - 1) // CHUNK_ELEMS
        n_rec = (rows + TILE_ROWS - 1) // TILE_ROWS * nch
        with torch.cuda.device(dev):
            st = torch.cuda.current_stream(dev).cuda_stream
            ptile_off = torch.empty(n_rec + 1, dtype=torch.int32, device=dev)
            call("bf16x_repack_count", *flat_args(f), out_f, in_f, r0, r1, ptile_off.data_ptr(), st)
            words = int(ptile_off[n_rec].item())
            layout = torch.empty((rows, row_bytes), dtype=torch.uint8, device=dev)
            precs = torch.zeros(max(words, 4), dtype=torch.int32, device=dev)
            call("bf16x_repack", *flat_args(f), out_f, in_f, r0, r1, ptile_off.data_ptr(), ptr(layout),
                 ptr(precs), st)
            _lib.check_device_status(dev.index)
        return cls(layout, ptile_off, precs, rows, in_f, out_f=out_f, row0=r0)

    # ------------------------------------------------------------ properties
    @property
    def device(self) -> torch.device:
        return self.layout.device

    @property
    def in_pad(self) -> int:
        return (self.in_f + CHUNK_ELEMS - 1) // CHUNK_ELEMS * CHUNK_ELEMS

    @property
    def row_bytes(self) -> int:
        return self.layout.shape[1]

    @property
    def n_patches(self) -> int:
        """Number of exact-delta patches (entries of all records)."""
        if self._n_patches is None:
            offs = self.ptile_off[:-1].long() + REC_HDR_WORD
            n_all = self.precs.view(torch.int16)[offs * 2 + 1].to(torch.int32) & 0xFFFF
            self._n_patches = int(n_all.sum().item())
        return self._n_patches

    def nbytes(self) -> int:
        """Bytes the fused kernels stream per full pass: layout + patch records + record offsets."""
        return self.layout.numel() + 4 * int(self.ptile_off[-1].item()) + 4 * self.ptile_off.numel()

    def bits_per_weight(self) -> float:
        return 8.0 * self.nbytes() / max(1, self.rows * self.in_f)

    # -------------------------------------------------------------- compute
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def decode(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """Exact bf16 weight rows [rows, in_f]."""
        if out is None:
            out = torch.empty((self.rows, self.in_f), dtype=torch.bfloat16, device=self.device)
        with torch.cuda.device(self.device):
            call("bf16x_resident_decode", ptr(self.layout), ptr(self.ptile_off), ptr(self.precs),
                 self.rows, self.in_f, ptr(out), out.stride(0), self._stream())
        return out

    def decode_rows(self, r0: int, r1: int) -> torch.Tensor:
        """Exact bf16 rows [r0, r1) of this weight (relative to its first row).
        Decoding starts at the 16-row tile holding r0: a tile's record covers
        its 16 rows, so the layout and record offsets are entered there."""
        r0, r1 = int(r0), int(r1)
        if not (0 <= r0 <= r1 <= self.rows):
            raise ValueError(f"row range [{r0}, {r1}) outside 0..{self.rows}")
        a = r0 // TILE_ROWS * TILE_ROWS
        out = torch.empty((r1 - a, self.in_f), dtype=torch.bfloat16, device=self.device)
        if r1 > a:
            nch = (self.in_f + CHUNK_ELEMS - 1) // CHUNK_ELEMS
            with torch.cuda.device(self.device):
                call("bf16x_resident_decode", self.layout.data_ptr() + a * self.row_bytes,
                     self.ptile_off.data_ptr() + 4 * (a // TILE_ROWS) * nch, ptr(self.precs),
                     r1 - a, self.in_f, ptr(out), out.stride(0), self._stream())
        return out[r0 - a:]

    def _prep_x(self, x2: torch.Tensor) -> torch.Tensor:
        """bf16 activations with a row pitch covering the padded columns (zeros)."""
        x2 = x2.to(torch.bfloat16)
        if (self.in_f % CHUNK_ELEMS == 0 and x2.is_contiguous() and x2.data_ptr() % 16 == 0):
            return x2
        xp = torch.zeros((x2.shape[0], self.in_pad), dtype=torch.bfloat16, device=self.device)
        xp[:, : self.in_f] = x2
        return xp

    def gemv(self, x: torch.Tensor, bias: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[b, n] = sum_k W[n, k] x[b, k] (+ bias) for a batch of <= 16 rows."""
        _lib.require_cuda(x, "x")
        x2 = x.reshape(-1, self.in_f)
        B = x2.shape[0]
        if B < 1 or B > GEMV_MAX_BATCH:
            raise ValueError(f"gemv takes 1..{GEMV_MAX_BATCH} rows of activations, got {B}")
        xp = self._prep_x(x2)
        if out is None:
            out = torch.empty((B, self.rows), dtype=out_dtype, device=self.device)
        ydt = _YDT[out.dtype]
        b = None
        if bias is not None:
            b = bias.to(device=self.device, dtype=torch.bfloat16).contiguous()
        dev = self.device
        if torch.cuda.current_device() == dev.index:
            self._launch_gemv(xp, B, b, out, ydt)
        else:
            with torch.cuda.device(dev):
                self._launch_gemv(xp, B, b, out, ydt)
        return out

    def _launch_gemv(self, xp, B, b, out, ydt):
        """bf16x_gemv on the current device and stream (the per-weight
        pointers looked up once)."""
        if self._wptrs is None:
            self._scratch_need = int(_lib.lib().bf16x_gemv_scratch_bytes(self.rows, self.in_f))
            self._wptrs = (self.layout.data_ptr(), self.ptile_off.data_ptr(), self.precs.data_ptr(),
                           self.tile_counters.data_ptr())
        st = torch.cuda.current_stream().cuda_stream
        ws = gemv_scratch(self.device, self._scratch_need, st)
        lay, pto, prc, cnt = self._wptrs
        _lib.check(_lib.lib().bf16x_gemv(lay, pto, prc, self.rows, self.in_f, xp.data_ptr(), B, xp.stride(0),
                                         ptr(b), out.data_ptr(), ydt, out.stride(0), cnt, ws.data_ptr(),
                                         ws.numel(), st), "bf16x_gemv")

    def gemv_peers(self, x: torch.Tensor, peers, ll_offset: int, out_total: int, y: torch.Tensor,
                   mode: int = 0, row0: int = 0, bias: torch.Tensor | None = None) -> torch.Tensor:
        """The fused decode+GEMV of this rank's weight whose epilogue does the
        tensor-parallel exchange over NVLink (``bf16x_gemv_peers``): every
        output goes, tagged with the launch's epoch, to the PeerGroup heap
        buffer at ``ll_offset`` of every rank, and each GPU builds ``y``
        ([batch, >= out_total], bf16 or fp32, this GPU's) from the words of
        its own copy.  mode 0: this weight is rows [row0, row0 + rows) of an
        out_total-row weight and y gets all rows (all-gather); mode 1: this
        weight is an input-column slice with every row (rows == out_total)
        and y gets the sum of all ranks' partials (all-reduce).  The heap
        buffer holds batch * out_total 64-bit words (mode 1: world times
        that); consecutive calls of a group must use different buffers."""
        _lib.require_cuda(x, "x")
        x2 = x.reshape(-1, self.in_f)
        B = x2.shape[0]
        if B < 1 or B > GEMV_MAX_BATCH:
            raise ValueError(f"gemv takes 1..{GEMV_MAX_BATCH} rows of activations, got {B}")
        if y.dim() != 2 or y.shape[0] < B or y.shape[1] < out_total or y.stride(1) != 1:
            raise ValueError(f"y must be [>= {B}, >= {out_total}] with unit column stride")
        xp = self._prep_x(x2)
        ydt = {torch.bfloat16: BF16X_DTYPE_BF16, torch.float32: BF16X_DTYPE_F32}[y.dtype]
        b = None if bias is None else bias.to(device=self.device, dtype=torch.bfloat16).contiguous()
        tables = getattr(self, "_peer_tables", None)
        if tables is None or tables[0] != (id(peers), ll_offset):
            tables = ((id(peers), ll_offset), peers.table(ll_offset))
            self._peer_tables = tables
        with torch.cuda.device(self.device):
            if self._scratch_need is None:
                self._scratch_need = int(_lib.lib().bf16x_gemv_scratch_bytes(self.rows, self.in_f))
            ws = gemv_scratch(self.device, self._scratch_need)
            call("bf16x_gemv_peers", ptr(self.layout), ptr(self.ptile_off), ptr(self.precs), self.rows, self.in_f,
                 ptr(xp), B, xp.stride(0), ptr(b), int(mode), tables[1], int(out_total), int(out_total), int(row0),
                 peers.world, peers.rank, ptr(y), ydt, y.stride(0), peers.state_ptr, ptr(self.tile_counters),
                 ptr(ws), ws.numel(), self._stream())
        return y[:B]

    def gemm(self, x: torch.Tensor, bias: torch.Tensor | None = None,
             out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[m, n] = sum_k W[n, k] x[m, k] (+ bias) on the tensor cores, any number of rows m."""
        _lib.require_cuda(x, "x")
        x2 = x.reshape(-1, self.in_f).to(torch.bfloat16)
        M = x2.shape[0]
        if not (x2.is_contiguous() and x2.data_ptr() % 16 == 0 and self.in_f % 8 == 0):
            ld = (self.in_f + 7) // 8 * 8
            xp = torch.zeros((M, ld), dtype=torch.bfloat16, device=self.device)
            xp[:, : self.in_f] = x2
            x2 = xp
        if out is None:
            out = torch.empty((M, self.rows), dtype=out_dtype, device=self.device)
        ydt = {torch.bfloat16: BF16X_DTYPE_BF16, torch.float32: BF16X_DTYPE_F32}[out.dtype]
        b = None if bias is None else bias.to(device=self.device, dtype=torch.bfloat16).contiguous()
        with torch.cuda.device(self.device):
            need = int(_lib.lib().bf16x_gemm_workspace_bytes(self.rows, self.in_f, M))
            ws = gemm_workspace(self.device, need) if need else None
            call("bf16x_gemm_ws", ptr(self.layout), ptr(self.ptile_off), ptr(self.precs), self.rows, self.in_f,
                 ptr(x2), M, x2.stride(0), ptr(b), ptr(out), ydt, out.stride(0),
                 ptr(ws) if ws is not None else None, ws.numel() if ws is not None else 0, self._stream())
        return out

    def linear(self, x: torch.Tensor, bias: torch.Tensor | None = None,
               out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """x[..., in_f] -> [..., rows]: the GEMV kernel for up to 16 rows of
        activations, the tensor-core GEMM above that."""
        od = out_dtype or (x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16)
        x2 = x.reshape(-1, self.in_f)
        M = x2.shape[0]
        if M <= GEMV_MAX_BATCH:
            y = self.gemv(x2, bias, out_dtype=od)
        else:
            y = self.gemm(x2, bias, out_dtype=od)
        return y.reshape(*x.shape[:-1], self.rows)


__all__ = ["ResidentWeight", "flat_on_device", "flat_args", "gemv_scratch", "gemm_workspace", "reset_workspaces",
           "GEMV_MAX_BATCH"]
