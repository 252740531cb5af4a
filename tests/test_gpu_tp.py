"""Tensor-parallel BF16X layers on 2 GPUs over NCCL: row-sharded (all-gather)
and column-sharded (all-reduce) layers against the CPU oracle within the 1e-3
relative-L2 gate, and the tensor-parallel decoder with packed shards.
Skipped with fewer than 2 GPUs."""
import datetime
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
        from bfloat16x_b200.tp import ColumnParallelBf16x, RowParallelBf16x
        from oracle import oracle
        from tests.gpu_util import bits_of, oracle_dict, rel_l2
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        w = synthetic_weight(1000, 2048, seed=3)
        wb = bits_of(w)
        p = oracle_dict(wb)
        res = []
        for M in (1, 7, 200):
            x = synthetic_activation(M, 2048, seed=M)
            ref = oracle.matmul_bf16w(x.float().numpy(), wb)
            row = RowParallelBf16x(p)
            y = row(x.cuda()).float().cpu().numpy()
            res.append(rel_l2(y, torch.from_numpy(ref).to(torch.bfloat16).float().numpy()) < 1e-3)
            col = ColumnParallelBf16x(w)
            y2 = col(x.cuda()).float().cpu().numpy()
            res.append(rel_l2(y2, torch.from_numpy(ref).to(torch.bfloat16).float().numpy()) < 1e-3)
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(res), res))
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_row_and_column_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1], r


def _decoder_worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        from bfloat16x_b200.llama_e2e import CONFIGS, LlamaModel, generate, pack_model
        cfg = CONFIGS["tiny"]
        prompt = torch.randint(0, cfg.vocab, (2, 24), generator=torch.Generator().manual_seed(2)).to(dev)
        model = LlamaModel(cfg, 64, dev, seed=4, tp=world, batch=2)
        pos0 = torch.zeros((), dtype=torch.long, device=dev)
        ref = model(prompt, pos0)
        pack_model(model)
        got = model(prompt, pos0)
        tok_g, _, _ = generate(model, prompt, 8, use_graph=True)
        tok_e, _, _ = generate(model, prompt, 8, use_graph=False)
        ok = [float((got - ref).norm() / ref.norm()) < 2e-2, bool(torch.equal(tok_g, tok_e)),
              tuple(tok_g.shape) == (8, 2)]
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(ok), ok))
    except Exception as e:
        q.put((rank, False, repr(e)))


# The tensor-parallel decoder with every shard BF16X-packed: prefill logits
# against its bf16 run, and CUDA-graph decode (NCCL collectives captured)
# against eager decode.
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_decoder_packed_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29800 + os.getpid() % 1000
    procs = [ctx.Process(target=_decoder_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1], r


def _peer_worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from bfloat16x_b200 import _lib
        from bfloat16x_b200.opqk_linear import bf16x_quantize
        from bfloat16x_b200.peer import PeerGroup
        from bfloat16x_b200.resident import ResidentWeight
        from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
        from bfloat16x_b200.tp import shard_bounds
        from tests.gpu_util import bits_of, oracle_dict, rel_l2
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        pg = PeerGroup(None, dev, heap_bytes=32 << 20)
        res = []
        # mode 0: row shards, every rank assembles all rows
        for (out_f, in_f), B, dt in [((1000, 2048), 1, torch.float32), ((4096, 4096), 8, torch.bfloat16),
                                     ((300, 1536), 3, torch.float32), ((2048, 1024), 16, torch.bfloat16)]:
            w = synthetic_weight(out_f, in_f, seed=out_f)
            r0, r1 = shard_bounds(out_f, world, rank, 16)
            rw = ResidentWeight.from_packed(oracle_dict(bits_of(w)), device=dev, row_range=(r0, r1))
            bufs = [pg.alloc(B * out_f * 8) for _ in range(2)]       # used alternately
            x = synthetic_activation(B, in_f, seed=B)
            ref = x.float() @ w.float().T
            ref_c = ref if dt == torch.float32 else ref.to(torch.bfloat16).float()
            for it in range(4):
                y = torch.full((B, out_f), float("nan"), dtype=dt, device=dev)
                rw.gemv_peers(x.to(dev), pg, bufs[it % 2], out_f, y, mode=0, row0=r0)
                torch.cuda.synchronize()
                got = y.float().cpu()
                res.append(bool(torch.isfinite(got).all()) and rel_l2(got.numpy(), ref_c.numpy()) < 1e-3)
            _lib.check_device_status(rank)
        # mode 1: column shards, every rank gets the sum of all partials
        for (out_f, in_f), B in [((1000, 2048), 1), ((4096, 4096), 5)]:
            w = synthetic_weight(out_f, in_f, seed=in_f + 1)
            c0, c1 = shard_bounds(in_f, world, rank, 256)
            rw = ResidentWeight.from_packed(bf16x_quantize(w[:, c0:c1].contiguous().to(dev), device=dev), device=dev)
            bufs = [pg.alloc(world * B * out_f * 8) for _ in range(2)]
            x = synthetic_activation(B, in_f, seed=B + 3)
            ref = x.float() @ w.float().T
            for it in range(3):
                y = torch.empty((B, out_f), dtype=torch.float32, device=dev)
                rw.gemv_peers(x[:, c0:c1].contiguous().to(dev), pg, bufs[it % 2], out_f, y, mode=1)
                torch.cuda.synchronize()
                res.append(rel_l2(y.cpu().numpy(), ref.numpy()) < 1e-3)
            _lib.check_device_status(rank)
        # the same launches captured in a CUDA graph and replayed: the epoch
        # lives in device memory, so replays keep the ranks in step
        out_f, in_f, B = 2048, 1024, 2
        w = synthetic_weight(out_f, in_f, seed=77)
        r0, r1 = shard_bounds(out_f, world, rank, 16)
        rw = ResidentWeight.from_packed(oracle_dict(bits_of(w)), device=dev, row_range=(r0, r1))
        x = synthetic_activation(B, in_f, seed=5).to(dev)
        bufs = [pg.alloc(B * out_f * 8) for _ in range(2)]
        ys = [torch.zeros((B, out_f), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for bo, yo in zip(bufs, ys):
                rw.gemv_peers(x, pg, bo, out_f, yo, mode=0, row0=r0)
            torch.cuda.synchronize(dev)
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for bo, yo in zip(bufs, ys):
                    rw.gemv_peers(x, pg, bo, out_f, yo, mode=0, row0=r0)
        torch.cuda.synchronize(dev)
        dist.barrier()
        ref = (x.float().cpu() @ w.float().T).to(torch.bfloat16).float()
        for _ in range(5):
            for yo in ys:
                yo.zero_()
            torch.cuda.synchronize(dev)
            g.replay()
            torch.cuda.synchronize(dev)
            for yo in ys:
                res.append(rel_l2(yo.float().cpu().numpy(), ref.numpy()) < 1e-3)
        _lib.check_device_status(rank)
        del g
        pg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(res), res))
    except Exception:
        import traceback
        q.put((rank, False, traceback.format_exc()))


# The GEMV whose epilogue exchanges outputs over NVLink (bf16x_gemv_peers):
# row shards gathered and column-shard partials summed on every rank, against
# the unsharded product, eager and replayed from a CUDA graph.
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemv_peers_allgather_2gpu():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 1000
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1], r


def _peer_layers_worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from bfloat16x_b200 import _lib
        from bfloat16x_b200.llama_e2e import (CONFIGS, LlamaModel, generate, pack_model, peer_heap_bytes,
                                              use_peer_collectives)
        from bfloat16x_b200.peer import PeerGroup
        from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
        from bfloat16x_b200.tp import ColumnParallelBf16x, RowParallelBf16x
        from oracle import oracle
        from tests.gpu_util import bits_of, oracle_dict, rel_l2
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        pg = PeerGroup(None, dev, heap_bytes=16 << 20)
        res = []
        w = synthetic_weight(1000, 2048, seed=3)
        wb = bits_of(w)
        p = oracle_dict(wb)
        row = RowParallelBf16x(p, peers=pg)
        col = ColumnParallelBf16x(w, peers=pg)
        for M in (1, 7, 16, 40):
            x = synthetic_activation(M, 2048, seed=M)
            ref = oracle.matmul_bf16w(x.float().numpy(), wb)
            ref16 = torch.from_numpy(ref).to(torch.bfloat16).float().numpy()
            for _ in range(2):
                y = row(x.cuda()).float().cpu().numpy()
                res.append(rel_l2(y, ref16) < 1e-3)
                y2 = col(x.cuda()).float().cpu().numpy()
                res.append(rel_l2(y2, ref16) < 1e-3)
        _lib.check_device_status(rank)
        # the tensor-parallel decoder: collectives in the fused GEMVs against NCCL
        cfg = CONFIGS["tiny"]
        prompt = torch.randint(0, cfg.vocab, (2, 24), generator=torch.Generator().manual_seed(2)).to(dev)
        model = LlamaModel(cfg, 64, dev, seed=4, tp=world, batch=2)
        pack_model(model)
        tok_n, _, _ = generate(model, prompt, 8, use_graph=True)
        pos = torch.tensor(24, dtype=torch.long, device=dev)
        lg_n = model(tok_n[:1].t().contiguous(), pos)
        pg2 = PeerGroup(None, dev, heap_bytes=peer_heap_bytes(model))
        use_peer_collectives(model, pg2)
        tok_p, _, _ = generate(model, prompt, 8, use_graph=True)
        lg_p = model(tok_n[:1].t().contiguous(), pos)
        res.append(bool(torch.equal(tok_p, tok_n)))
        res.append(float((lg_p - lg_n).norm() / lg_n.norm()) < 1e-2)
        _lib.check_device_status(rank)
        torch.cuda.synchronize()
        pg2.close()
        pg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(res), res))
    except Exception:
        import traceback
        q.put((rank, False, traceback.format_exc()))


# Row- and column-parallel layers whose all-gather / all-reduce run inside
# the fused GEMV (PeerGroup), and the tensor-parallel decoder with its
# collectives moved there, against NCCL.
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_layers_and_decoder_peer_collectives_2gpu():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29200 + os.getpid() % 1000
    procs = [ctx.Process(target=_peer_layers_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1], r
