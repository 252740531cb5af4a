"""Tensor-parallel decoder on the host: two gloo ranks build their shards of
the small Llama-style model on the CPU (bf16 weights, plain torch linears)
and their logits -- prefill and one decode step, through the all-reduce of
o_proj/down_proj and the all-gather of lm_head -- match the unsharded model
built from the same seed in each rank."""
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from bfloat16x_b200.llama_e2e import CONFIGS, LlamaModel
        torch.set_num_threads(2)
        cfg = CONFIGS["tiny"]
        batch, P = 2, 12
        ids = torch.randint(0, cfg.vocab, (batch, P), generator=torch.Generator().manual_seed(5))
        full = LlamaModel(cfg, 32, "cpu", seed=3, tp=1, batch=batch)
        shard = LlamaModel(cfg, 32, "cpu", seed=3, tp=world, batch=batch)
        pos0 = torch.zeros((), dtype=torch.long)
        ref = full(ids, pos0)
        got = shard(ids, pos0)
        tok = ref.argmax(-1, keepdim=True)
        ref2 = full(tok, pos0 + P)
        got2 = shard(tok, pos0 + P)
        rel = lambda a, b: float((a - b).norm() / b.norm())
        q.put((rank, tuple(got.shape) == (batch, cfg.vocab), rel(got, ref), rel(got2, ref2),
               shard.cache_k.shape[3] == cfg.kv_heads // world))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


def test_tp2_decoder_matches_unsharded_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 5, r
        _, shape_ok, e1, e2, kv_ok = r
        assert shape_ok and kv_ok, r
        assert e1 < 2e-2 and e2 < 2e-2, r      # bf16 partial sums rounded before the reduction
