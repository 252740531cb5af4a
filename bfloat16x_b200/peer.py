"""Device memory shared over NVLink by the ranks of one node, for the fused
decode+GEMV whose epilogue sends every output straight into every rank's
exchange buffer (``bf16x_gemv_peers``): the row-sharded layer's all-gather,
or the column-sharded layer's all-reduce, happens inside the kernel instead
of in a separate NCCL call.

``PeerGroup`` is collective: every rank of the process group builds one with
the same heap size.  Each rank allocates one device buffer, exports it
(CUDA IPC), exchanges the handles over the process group's host side
(``all_gather_object``) and maps every peer's buffer.  The buffer holds a
header -- this rank's launch state (finished-CTA count, epoch of the last
launch) -- followed by a zeroed heap carved out by ``alloc`` at the same
offsets on every rank, so an offset names "the same" buffer everywhere.

Rules the kernels rely on (each stated where it is enforced):
* the collective GEMVs of one group run in the same order on every rank, on
  one stream per rank (the epoch of the k-th launch is k on every rank);
* a heap buffer written by one collective GEMV is not written again by the
  very next one (consecutive layers use different buffers), so a rank that
  runs ahead never overwrites rows another rank is still reading;
* after a device error (a timed-out wait), ``reset`` clears the state and
  the heap on every rank before the group is used again.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call

HEADER_BYTES = 4096          # state (2 words) at 0
ALIGN = 256
MAX_RANKS = 8


class PeerGroup:
    """One NVLink-shared buffer per rank of ``group`` (see the module doc)."""

    def __init__(self, group=None, device=None, heap_bytes: int = 1 << 20):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"PeerGroup spans at most {MAX_RANKS} GPUs (one NVSwitch domain)")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.heap_bytes = int(heap_bytes)
        self.buf = torch.zeros(HEADER_BYTES + self.heap_bytes, dtype=torch.uint8, device=self.device)
        # Every step below is taken by every rank, and a failure on any rank
        # (no IPC on this node, say) raises on all of them at the same point,
        # so no rank is left waiting in a collective.
        try:
            mine = self._export(self.buf.data_ptr())
        except _lib.Bf16xError as e:
            mine = ("error", str(e))
        entries = [None] * self.world
        dist.all_gather_object(entries, mine, group=group)
        bad = [e[1] for e in entries if e[0] == "error"]
        if bad:
            raise _lib.Bf16xError(f"PeerGroup: a rank could not export its buffer: {bad[0]}")
        self._imported = []
        self.ptrs = []                                   # base of every rank's buffer, in this address space
        err = ""
        for q, (h, off) in enumerate(entries):
            if q == self.rank:
                self.ptrs.append(self.buf.data_ptr())
                continue
            try:
                base = self._import(h)
            except _lib.Bf16xError as e:
                err = str(e)
                break
            self._imported.append(base)
            self.ptrs.append(base + off)
        errs = [None] * self.world
        dist.all_gather_object(errs, err, group=group)
        if any(errs):
            for base in self._imported:
                self._close(base)
            self._imported = []
            raise _lib.Bf16xError(f"PeerGroup: a rank could not map its peers' buffers: {next(e for e in errs if e)}")
        self._next = HEADER_BYTES
        self._sync()
        dist.barrier(group=group)

    def _sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    # ---- the CUDA IPC calls (one place, so host tests can replace them) ----
    @staticmethod
    def _export(ptr: int):
        n = int(_lib.lib().bf16x_peer_handle_bytes())
        h = (ctypes.c_char * n)()
        off = ctypes.c_int64(0)
        call("bf16x_peer_export", ptr, h, ctypes.byref(off))
        return bytes(h), int(off.value)

    @staticmethod
    def _import(handle: bytes) -> int:
        base = ctypes.c_void_p(0)
        call("bf16x_peer_import", handle, ctypes.byref(base))
        return int(base.value)

    @staticmethod
    def _close(base: int) -> None:
        call("bf16x_peer_close", base)

    # ---- heap --------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        """Offset of a new heap buffer of nbytes (256-byte aligned).  Every
        rank must make the same sequence of calls."""
        off = self._next
        end = off + (int(nbytes) + ALIGN - 1) // ALIGN * ALIGN
        if end > HEADER_BYTES + self.heap_bytes:
            raise _lib.Bf16xError(f"PeerGroup heap exhausted ({self.heap_bytes} bytes)")
        self._next = end
        return off

    def local(self, offset: int, shape, dtype: torch.dtype) -> torch.Tensor:
        """This rank's copy of the heap buffer at `offset`, as a tensor."""
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return self.buf[offset:offset + nbytes].view(dtype).view(*shape)

    def table(self, offset: int):
        """Device addresses of the heap buffer at `offset` on every rank (a
        C array of pointers, rank order)."""
        return (ctypes.c_void_p * self.world)(*[p + offset for p in self.ptrs])

    @property
    def state_ptr(self) -> int:
        return self.ptrs[self.rank]

    # ---- lifetime ----------------------------------------------------------
    def reset(self) -> None:
        """Zero this rank's state and heap, collectively (after a device error)."""
        self._sync()
        dist.barrier(group=self.group)
        self.buf.zero_()
        self._sync()
        dist.barrier(group=self.group)

    def close(self) -> None:
        """Unmap the peers' buffers, collectively (no collective GEMV may be in
        flight on any rank)."""
        self._sync()
        dist.barrier(group=self.group)
        for base in self._imported:
            self._close(base)
        self._imported = []
        dist.barrier(group=self.group)


__all__ = ["PeerGroup", "HEADER_BYTES"]
