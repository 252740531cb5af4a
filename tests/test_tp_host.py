"""Host logic of the tensor-parallel layers on CPU: shard bounds, and the
all-gather / all-reduce assembly run by two gloo ranks with a plain CPU
matmul standing in for the per-rank fused kernel."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bfloat16x_b200.tp import ColumnParallel, RowParallel, shard_bounds


@pytest.mark.parametrize("n,world,align", [(4096, 2, 16), (4096, 8, 16), (14336, 8, 256), (300, 4, 16),
                                           (17, 2, 16), (8, 4, 16), (128256, 8, 16), (4096, 3, 256)])
def test_shard_bounds_cover(n, world, align):
    b = [shard_bounds(n, world, r, align) for r in range(world)]
    assert b[0][0] == 0 and b[-1][1] == n
    for (l0, h0), (l1, h1) in zip(b, b[1:]):
        assert h0 == l1 and l0 <= h0
    for l, h in b[:-1]:
        assert l % align == 0 and h % align == 0
    sizes = [h - l for l, h in b]
    assert max(sizes[:-1] or [0]) - min(sizes[:-1] or [0]) <= align


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(0)
        out_f, in_f = 300, 512
        W = torch.randn(out_f, in_f, generator=g)
        x = torch.randn(5, in_f, generator=g)
        r0, r1 = shard_bounds(out_f, world, rank, 16)
        row = RowParallel(lambda t: t @ W[r0:r1].T, out_f)
        y = row(x)
        ok_row = torch.allclose(y, x @ W.T, rtol=1e-5, atol=1e-5)
        c0, c1 = shard_bounds(in_f, world, rank, 256)
        col = ColumnParallel(lambda t: t @ W[:, c0:c1].T, in_f)
        y2 = col(x)
        ok_col = torch.allclose(y2, x @ W.T, rtol=1e-4, atol=1e-4)
        # a row-sharded layer feeding a column-sharded one with no gather between
        W2 = torch.randn(64, out_f, generator=g)
        up = RowParallel(lambda t: t @ W[r0:r1].T, out_f, gather=False)
        down = ColumnParallel(lambda t: t @ W2[:, r0:r1].T, out_f, input_is_sharded=True, align=16)
        y3 = down(up(x))
        ok_pair = torch.allclose(y3, (x @ W.T) @ W2.T, rtol=1e-4, atol=1e-3)
        q.put((rank, bool(ok_row), bool(ok_col), bool(ok_pair)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2])
def test_row_and_column_parallel_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1:] == (True, True, True), r


def _peer_worker(rank, world, port, q, fail_rank):
    """PeerGroup's host logic over gloo on CPU, with the CUDA IPC calls
    replaced by stand-ins (a handle is the rank's buffer address)."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from bfloat16x_b200 import _lib
        from bfloat16x_b200.peer import HEADER_BYTES, PeerGroup

        closed = []

        def export(ptr):
            if rank == fail_rank:
                raise _lib.Bf16xError("no IPC here")
            return (int(ptr).to_bytes(8, "little") + bytes(56), 64)

        PeerGroup._export = staticmethod(export)
        PeerGroup._import = staticmethod(lambda h: int.from_bytes(h[:8], "little") + 1000)
        PeerGroup._close = staticmethod(lambda base: closed.append(base))
        try:
            pg = PeerGroup(None, torch.device("cpu"), heap_bytes=1 << 16)
        except _lib.Bf16xError as e:
            dist.barrier()
            dist.destroy_process_group()
            q.put((rank, fail_rank >= 0, "failed on every rank: " + str(e)))
            return
        ok = [pg.world == world, pg.rank == rank, len(pg.ptrs) == world]
        ok.append(pg.ptrs[rank] == pg.buf.data_ptr())
        a, b = pg.alloc(100), pg.alloc(3000)
        ok += [a == HEADER_BYTES, b == HEADER_BYTES + 256, b % 256 == 0]
        t = pg.table(b)
        ok += [t[rank] == pg.buf.data_ptr() + b, pg.state_ptr == pg.buf.data_ptr()]
        # every rank's view of every buffer: its base (+ the stand-in mapping) + the same offset
        bases = [None] * world
        dist.all_gather_object(bases, pg.buf.data_ptr())
        ok += [t[q_] == (bases[q_] if q_ == rank else bases[q_] + 1000 + 64) + b for q_ in range(world)]
        ok.append(tuple(pg.local(b, (3, 250), torch.float32).shape) == (3, 250))
        try:
            pg.alloc(1 << 20)
            ok.append(False)
        except _lib.Bf16xError:
            ok.append(True)
        pg.close()
        ok.append(len(closed) == world - 1)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, fail_rank < 0 and all(ok), ok))
    except Exception:
        import traceback
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_peer_group_host_logic_gloo(fail_rank):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200 + (fail_rank + 1) * 7
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1], r


def _dead_peer_worker(rank, world, port, q):
    """Rank 1 leaves before building the PeerGroup (between steps, nothing in
    flight); rank 0 must get an error from its next collective, not hang."""
    import datetime
    import time
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        from bfloat16x_b200 import _lib
        from bfloat16x_b200.peer import PeerGroup
        PeerGroup._export = staticmethod(lambda ptr: (int(ptr).to_bytes(8, "little") + bytes(56), 0))
        PeerGroup._import = staticmethod(lambda h: int.from_bytes(h[:8], "little"))
        PeerGroup._close = staticmethod(lambda base: None)
        if rank == 1:
            q.put((rank, True, "left"))
            q.close()
            q.join_thread()            # the message is out before the process vanishes
            os._exit(0)
        t0 = time.time()
        try:
            PeerGroup(None, torch.device("cpu"), heap_bytes=4096)
            q.put((rank, False, "PeerGroup built without its peer"))
        except (RuntimeError, _lib.Bf16xError) as e:
            q.put((rank, time.time() - t0 < 60, f"raised after {time.time() - t0:.1f} s: {type(e).__name__}"))
    except Exception:
        import traceback
        q.put((rank, False, traceback.format_exc()))


def test_peer_group_dead_rank_raises():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29950 + os.getpid() % 40
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in res:
        assert r[1], r
