"""Tensor-parallel BF16X linears over ``torch.distributed`` (NCCL across the
GPUs of one node; any backend for the host logic).

A BF16X weight shards naturally by output rows: every rank holds rows
[r0, r1) in the resident layout (built straight from the full flat dict with
``bf16x_repack``'s row range, no re-quantisation) and runs the fused kernels
on them with no communication.  The only exchange is between layers:

* ``RowParallelBf16x``    -- output rows sharded; y shards are all-gathered
  into the full [..., out_f] (or returned local with ``gather=False``, for a
  following column-parallel layer).
* ``ColumnParallelBf16x`` -- input columns sharded (the Megatron pairing for
  o_proj / down_proj): each rank multiplies its column slice of W by its
  slice of x and the partial outputs are all-reduced (fp32 sum).

Shard bounds are multiples of 16 rows (the resident layout's tile) or of 256
columns (its chunk) whenever the size allows, so no tile or chunk straddles
two ranks.  ``RowParallel`` / ``ColumnParallel`` hold the collective logic
around any local compute callable.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist
import torch.nn as nn


def shard_bounds(n: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """Contiguous share [lo, hi) of n items for `rank` of `world`: units of
    `align` items dealt as evenly as possible, the remainder to the last rank."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    units = n // align
    base, extra = divmod(units, world)
    lo = align * (base * rank + min(rank, extra))
    hi = align * (base * (rank + 1) + min(rank + 1, extra))
    if rank == world - 1:
        hi = n
    return lo, hi


class RowParallel(nn.Module):
    """y[..., out_f] from per-rank row shards: local(x) gives [..., r1 - r0]
    for this rank's rows, then an all-gather assembles the full output."""

    def __init__(self, local: Callable[[torch.Tensor], torch.Tensor], out_f: int, group=None,
                 gather: bool = True, align: int = 16):
        super().__init__()
        self.local = local
        self.out_f = int(out_f)
        self.group = group
        self.gather = gather
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.bounds = [shard_bounds(self.out_f, self.world, r, align) for r in range(self.world)]
        self.max_rows = max(h - l for l, h in self.bounds)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x)
        if not self.gather or self.world == 1:
            return y
        lead = y.shape[:-1]
        y2 = y.reshape(-1, y.shape[-1])
        m = y2.shape[0]
        # equal-size pieces for the collective: pad every shard to max_rows
        piece = torch.zeros((m, self.max_rows), dtype=y2.dtype, device=y2.device)
        piece[:, : y2.shape[1]] = y2
        buf = torch.empty((self.world * m, self.max_rows), dtype=y2.dtype, device=y2.device)
        dist.all_gather_into_tensor(buf, piece.contiguous(), group=self.group)
        buf = buf.view(self.world, m, self.max_rows)
        parts = [buf[r, :, : h - l] for r, (l, h) in enumerate(self.bounds)]
        return torch.cat(parts, dim=1).reshape(*lead, self.out_f)


class ColumnParallel(nn.Module):
    """y[..., out_f] = sum over ranks of local(x[..., c0:c1]) (all-reduced in
    fp32), each rank holding W[:, c0:c1]."""

    def __init__(self, local: Callable[[torch.Tensor], torch.Tensor], in_f: int, group=None,
                 input_is_sharded: bool = False, align: int = 256):
        super().__init__()
        self.local = local
        self.in_f = int(in_f)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.c0, self.c1 = shard_bounds(self.in_f, self.world, self.rank, align)
        self.input_is_sharded = input_is_sharded

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xs = x if self.input_is_sharded else x[..., self.c0:self.c1]
        y = self.local(xs.contiguous())
        if self.world == 1:
            return y
        acc = y.float().contiguous()
        dist.all_reduce(acc, op=dist.ReduceOp.SUM, group=self.group)
        return acc.to(y.dtype)


class RowParallelBf16x(RowParallel):
    """Rows [r0, r1) of a BF16X dict resident on this rank's GPU.

    With ``peers`` (a PeerGroup over the same ranks), up to 16 rows of
    activations take the fused decode+GEMV whose epilogue sends each rank's
    output rows to every rank over NVLink and assembles the full output on
    each (``ResidentWeight.gemv_peers``, mode 0): no separate all-gather.
    More rows take the GEMM and NCCL."""

    def __init__(self, packed: dict, bias: torch.Tensor | None = None, group=None, gather: bool = True,
                 device=None, peers=None, max_batch: int = 16):
        from .resident import ResidentWeight
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        out_f = int(packed["out_f"])
        r0, r1 = shard_bounds(out_f, world, rank, 16)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        # a rank can own no rows when out_f < 16 * world
        self_rw = ResidentWeight.from_packed(packed, device=dev, row_range=(r0, r1)) if r1 > r0 else None
        b = None if bias is None else bias[r0:r1].detach().to(dev, torch.bfloat16).contiguous()

        def local(x):
            if self_rw is None:
                return torch.empty((*x.shape[:-1], 0), dtype=x.dtype, device=x.device)
            return self_rw.linear(x, b)

        super().__init__(local, out_f, group, gather, 16)
        self.resident = self_rw
        self.rows = (r0, r1)
        self.peers = peers if (gather and world > 1) else None
        self._bias = b
        if self.peers is not None:
            if any(h <= l for l, h in self.bounds):
                raise ValueError("the in-kernel all-gather needs rows on every rank (out_f >= 16 * world)")
            self.max_batch = int(max_batch)
            # two exchange buffers used alternately, so consecutive calls of
            # this layer never share one (the rule of bf16x_gemv_peers)
            self._lloff = [peers.alloc(self.max_batch * out_f * 8) for _ in range(2)]
            self._turn = 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.peers is None:
            return super().forward(x)
        x2 = x.reshape(-1, x.shape[-1])
        B = x2.shape[0]
        if B > self.max_batch:
            return super().forward(x)
        od = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16
        off = self._lloff[self._turn]
        self._turn ^= 1
        y = torch.empty((B, self.out_f), dtype=od, device=x.device)
        self.resident.gemv_peers(x2, self.peers, off, self.out_f, y, mode=0, row0=self.rows[0], bias=self._bias)
        return y.reshape(*x.shape[:-1], self.out_f)


class ColumnParallelBf16x(ColumnParallel):
    """Columns [c0, c1) of a bf16 weight, BF16X-packed on this rank's GPU.
    The bias, if any, is added once after the reduction.

    With ``peers``, up to 16 rows of activations take the fused decode+GEMV
    whose epilogue sends this rank's fp32 partial outputs to its slot of every
    rank's exchange buffer over NVLink, and each rank sums the slots in rank
    order (the same sum everywhere) inside the same kernel: no NCCL
    all-reduce (``ResidentWeight.gemv_peers``, mode 1)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, group=None,
                 input_is_sharded: bool = False, device=None, peers=None, max_batch: int = 16):
        from .opqk_linear import bf16x_quantize
        from .resident import ResidentWeight
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        in_f = weight.shape[1]
        c0, c1 = shard_bounds(in_f, world, rank, 256)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        p = bf16x_quantize(weight[:, c0:c1].to(dev, torch.bfloat16).contiguous(), device=dev)
        rw = ResidentWeight.from_packed(p, device=dev)

        def local(x):
            return rw.linear(x, None, out_dtype=torch.float32)

        super().__init__(local, in_f, group, input_is_sharded, 256)
        self.resident = rw
        self.bias = None if bias is None else bias.detach().to(dev, torch.bfloat16)
        self.peers = peers if world > 1 else None
        if self.peers is not None:
            self.max_batch = int(max_batch)
            self.out_f = int(weight.shape[0])
            self._lloff = [peers.alloc(world * self.max_batch * self.out_f * 8) for _ in range(2)]
            self._turn = 0

    def _peer_sum(self, x: torch.Tensor) -> torch.Tensor:
        xs = x if self.input_is_sharded else x[..., self.c0:self.c1]
        x2 = xs.reshape(-1, xs.shape[-1]).contiguous()
        B = x2.shape[0]
        off = self._lloff[self._turn]
        self._turn ^= 1
        y = torch.empty((B, self.out_f), dtype=torch.float32, device=x2.device)
        self.resident.gemv_peers(x2, self.peers, off, self.out_f, y, mode=1)
        return y.reshape(*x.shape[:-1], self.out_f)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.peers is not None and x.numel() // x.shape[-1] <= self.max_batch:
            y = self._peer_sum(x)
        else:
            y = super().forward(x)
        if self.bias is not None:
            y = y + self.bias.float()
        return y.to(x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.bfloat16)


__all__ = ["shard_bounds", "RowParallel", "ColumnParallel", "RowParallelBf16x", "ColumnParallelBf16x"]
