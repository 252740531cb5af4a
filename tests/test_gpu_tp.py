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
