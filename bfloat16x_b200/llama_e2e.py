"""End-to-end decoder for the BF16X path: a Llama-style model whose linear
layers (attention and MLP projections and lm_head) are BF16X-packed and run
through the fused decode+GEMV (up to 16 tokens) and decode+GEMM (more tokens)
kernels.

It exists to measure the hot path inside a model: ms per generated token
against the same model with plain bf16 weights (cuBLAS), after a prompt
prefill, for the two decoder configurations of the benchmark (``CONFIGS``).
Weights are random N(0, 0.02) (no checkpoints), drawn per weight from a
seeded generator so that every tensor-parallel degree builds the same model;
attention uses torch's scaled_dot_product_attention over a static KV cache,
so one decode step has static shapes and is replayed as a CUDA graph.

Tensor parallelism (``tp`` ranks of a process group, Megatron pairing): each
rank holds its query/key/value heads and its slice of the MLP's hidden units
(rows of the fused qkv and gate/up weights), the matching input columns of
o_proj and down_proj (partial outputs summed by an all-reduce) and a vocab
slice of lm_head (logits all-gathered); embeddings and norms are replicated.

"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from . import _lib


@dataclass
class LlamaConfig:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 500000.0
    eps: float = 1e-5


CONFIGS = {
    # 1B-class Llama-style decoder (hidden 2048, 24 layers, GQA 16/8, vocab 73448)
    "1b": LlamaConfig(hidden=2048, layers=24, heads=16, kv_heads=8, head_dim=128, ffn=6144, vocab=73448),
    # 8B Llama-3-style decoder (hidden 4096, 32 layers, GQA 32/8, vocab 128256)
    "8b": LlamaConfig(hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256),
    # a small one for tests
    "tiny": LlamaConfig(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000),
}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class RMSNorm(nn.Module):
    def __init__(self, n: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n, dtype=torch.bfloat16), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        if x.is_cuda:
            return self.add_forward(x, None)[1]
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)

    def add_forward(self, x, delta):
        """(h, norm(h)) with h = x + delta (delta may be None): one kernel on
        the GPU (bf16x_add_rmsnorm), the framework ops on the CPU."""
        if not x.is_cuda:
            h = x if delta is None else x + delta
            return h, self.forward(h)
        x = x.contiguous()
        n = x.shape[-1]
        y = torch.empty_like(x)
        h = x if delta is None else torch.empty_like(x)
        d = None if delta is None else delta.to(x.dtype).contiguous()
        _lib.call("bf16x_add_rmsnorm", x.data_ptr(), None if d is None else d.data_ptr(), self.weight.data_ptr(),
                  float(self.eps), x.numel() // n, n, None if d is None else h.data_ptr(), y.data_ptr(), _stream(x))
        return h, y


def _rope_tables(head_dim: int, max_pos: int, theta: float, device):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    t = torch.arange(max_pos, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return torch.cos(f), torch.sin(f)


def _apply_rope(x, cos, sin):
    # x [B, T, H, D]; cos/sin [T, D/2]
    x1, x2 = x[..., 0::2].float(), x[..., 1::2].float()
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    y = torch.stack((x1 * c - x2 * s, x1 * s + x2 * c), dim=-1).flatten(-2)
    return y.to(x.dtype)


def _rand_weight(out_f: int, in_f: int, seed: int, device) -> torch.Tensor:
    """bf16 N(0, 0.02) weight [out_f, in_f] from its own seeded generator."""
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(out_f, in_f, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)


def _linear_from(w: torch.Tensor) -> nn.Linear:
    lin = nn.Linear(w.shape[1], w.shape[0], bias=False, device=w.device, dtype=w.dtype)
    lin.weight.data = w.contiguous()
    return lin


class ColumnShard(nn.Module):
    """The input-column slice of a linear: this rank's partial outputs,
    summed over the group.  By default an fp32 NCCL all-reduce; once packed
    and given a PeerGroup (``use_peer_collectives``), up to 16 tokens take the
    fused decode+GEMV that sends the fp32 partials to this rank's slot of
    every rank's exchange buffer over NVLink and sums the slots in rank order
    (the same sum on every rank) inside the same kernel."""

    def __init__(self, lin: nn.Module, group=None, tp: int = 1):
        super().__init__()
        self.lin, self.group, self.tp = lin, group, tp
        self.peers = None

    def attach_peers(self, peers, max_batch: int) -> None:
        self.peers = peers
        self.max_batch = max_batch
        self.out_f = self.lin.out_features
        self._lloff = peers.alloc(peers.world * max_batch * self.out_f * 8)
        self._y = torch.empty((max_batch, self.out_f), dtype=torch.bfloat16, device=peers.device)

    def forward(self, x):
        if self.peers is not None and x.numel() // x.shape[-1] <= self.max_batch:
            x2 = x.reshape(-1, x.shape[-1])
            y = self.lin.rw.gemv_peers(x2, self.peers, self._lloff, self.out_f, self._y, mode=1)
            return y.to(x.dtype).reshape(*x.shape[:-1], self.out_f)
        y = self.lin(x)
        if self.tp == 1:
            return y
        acc = y.float()
        dist.all_reduce(acc, group=self.group)
        return acc.to(y.dtype)


class VocabShard(nn.Module):
    """Rows [r0, r1) of lm_head on this rank; the logits of all ranks are
    all-gathered (equal pieces of ``piece`` rows, the last one padded)."""

    def __init__(self, lin: nn.Module, vocab: int, piece: int, group=None, tp: int = 1):
        super().__init__()
        self.lin, self.vocab, self.piece, self.group, self.tp = lin, vocab, piece, group, tp
        self.peers = None

    def attach_peers(self, peers, max_batch: int) -> None:
        """Logits gathered inside the fused GEMV (every rank's vocab rows
        stored into every rank's logits buffer over NVLink)."""
        self.peers = peers
        self.max_batch = max_batch
        self._lloff = peers.alloc(max_batch * self.vocab * 8)
        self._y = torch.empty((max_batch, self.vocab), dtype=torch.bfloat16, device=peers.device)

    def forward(self, x):
        if self.peers is not None and x.numel() // x.shape[-1] <= self.max_batch:
            x2 = x.reshape(-1, x.shape[-1])
            pg = self.peers
            y = self.lin.rw.gemv_peers(x2, pg, self._lloff, self.vocab, self._y, mode=0, row0=pg.rank * self.piece)
            return y.reshape(*x.shape[:-1], self.vocab)
        y = self.lin(x)
        if self.tp == 1:
            return y
        y2 = y.reshape(-1, y.shape[-1])
        buf = torch.zeros((y2.shape[0], self.piece), dtype=y2.dtype, device=y2.device)
        buf[:, : y2.shape[1]] = y2
        out = torch.empty((self.tp * y2.shape[0], self.piece), dtype=y2.dtype, device=y2.device)
        dist.all_gather_into_tensor(out, buf, group=self.group)
        full = out.view(self.tp, y2.shape[0], self.piece).permute(1, 0, 2).reshape(y2.shape[0], -1)
        return full[:, : self.vocab].reshape(*y.shape[:-1], self.vocab)


def _vocab_piece(vocab: int, tp: int) -> int:
    return (vocab + tp - 1) // tp


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig, layer: int, seed: int, device, tp: int = 1, rank: int = 0, group=None):
        super().__init__()
        if cfg.heads % tp or cfg.kv_heads % tp:
            raise ValueError("heads and kv_heads must divide by the tensor-parallel degree")
        self.cfg, self.tp = cfg, tp
        self.h, self.kvh, self.d = cfg.heads // tp, cfg.kv_heads // tp, cfg.head_dim
        d, H, KV = cfg.head_dim, cfg.heads, cfg.kv_heads
        # q, k and v projections as one [q; k; v] weight (this rank's heads): one GEMV per step
        w = _rand_weight((H + 2 * KV) * d, cfg.hidden, seed + 1000 * layer + 1, device)
        q = w[rank * self.h * d:(rank + 1) * self.h * d]
        k = w[H * d + rank * self.kvh * d:H * d + (rank + 1) * self.kvh * d]
        v = w[(H + KV) * d + rank * self.kvh * d:(H + KV) * d + (rank + 1) * self.kvh * d]
        self.qkv_proj = _linear_from(torch.cat([q, k, v]))
        del w
        w = _rand_weight(cfg.hidden, H * d, seed + 1000 * layer + 2, device)
        self.o_proj = ColumnShard(_linear_from(w[:, rank * self.h * d:(rank + 1) * self.h * d]), group, tp)

    def forward(self, x, pos0, cache_k, cache_v, cos, sin, mask, tables=None):
        B, T, _ = x.shape
        qkv = self.qkv_proj(x)
        nq, nk = self.h * self.d, self.kvh * self.d
        if x.is_cuda and tables is not None:
            # rotary embedding of q and k and the cache write of k and v: one kernel
            qkv = qkv.contiguous()
            q = torch.empty((B, T, self.h, self.d), dtype=qkv.dtype, device=x.device)
            cos_t, sin_t = tables
            _lib.call("bf16x_rope_qkv", qkv.data_ptr(), B * T, T, self.h, self.kvh, self.d, pos0.data_ptr(),
                      cos_t.data_ptr(), sin_t.data_ptr(), q.data_ptr(), cache_k.data_ptr(), cache_v.data_ptr(),
                      cache_k.stride(0), cache_k.shape[1], _stream(x))
        else:
            q = qkv[..., :nq].reshape(B, T, self.h, self.d)
            k = qkv[..., nq:nq + nk].reshape(B, T, self.kvh, self.d)
            v = qkv[..., nq + nk:].reshape(B, T, self.kvh, self.d)
            q, k = _apply_rope(q, cos, sin), _apply_rope(k, cos, sin)
            # write this step's keys/values at positions pos0 .. pos0+T-1
            idx = pos0 + torch.arange(T, device=x.device)
            cache_k.index_copy_(1, idx, k)
            cache_v.index_copy_(1, idx, v)
        # grouped-query attention over the whole static cache (masked)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), cache_k.transpose(1, 2), cache_v.transpose(1, 2),
                                           attn_mask=mask, enable_gqa=True)
        return self.o_proj(o.transpose(1, 2).reshape(B, T, self.h * self.d))


class MLP(nn.Module):
    def __init__(self, cfg: LlamaConfig, layer: int, seed: int, device, tp: int = 1, rank: int = 0, group=None):
        super().__init__()
        if cfg.ffn % tp:
            raise ValueError("ffn must divide by the tensor-parallel degree")
        self.ffn = cfg.ffn // tp
        f0, f1 = rank * self.ffn, (rank + 1) * self.ffn
        # gate and up projections as one [gate; up] weight (this rank's hidden units)
        w = _rand_weight(2 * cfg.ffn, cfg.hidden, seed + 1000 * layer + 3, device)
        self.gate_up_proj = _linear_from(torch.cat([w[f0:f1], w[cfg.ffn + f0:cfg.ffn + f1]]))
        del w
        w = _rand_weight(cfg.hidden, cfg.ffn, seed + 1000 * layer + 4, device)
        self.down_proj = ColumnShard(_linear_from(w[:, f0:f1]), group, tp)

    def forward(self, x):
        gu = self.gate_up_proj(x)
        if gu.is_cuda:
            gu = gu.contiguous()
            act = torch.empty((*gu.shape[:-1], self.ffn), dtype=gu.dtype, device=gu.device)
            _lib.call("bf16x_silu_mul", gu.data_ptr(), gu.numel() // (2 * self.ffn), self.ffn, act.data_ptr(),
                      _stream(gu))
            return self.down_proj(act)
        return self.down_proj(F.silu(gu[..., :self.ffn]) * gu[..., self.ffn:])


class Block(nn.Module):
    def __init__(self, cfg: LlamaConfig, layer: int, seed: int, device, tp: int = 1, rank: int = 0, group=None):
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.eps)
        self.self_attn = Attention(cfg, layer, seed, device, tp, rank, group)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.eps)
        self.mlp = MLP(cfg, layer, seed, device, tp, rank, group)

    def forward(self, x, pos0, ck, cv, cos, sin, mask):
        x = x + self.self_attn(self.input_layernorm(x), pos0, ck, cv, cos, sin, mask)
        return x + self.mlp(self.post_attention_layernorm(x))


class LlamaModel(nn.Module):
    """Llama-style decoder with a static KV cache of ``max_seq`` positions for
    ``batch`` sequences; ``tp`` > 1 builds this rank's shard (``group``: the
    tensor-parallel process group, default the world)."""

    def __init__(self, cfg: LlamaConfig, max_seq: int, device, seed: int = 0, tp: int = 1, group=None,
                 batch: int = 1):
        super().__init__()
        device = torch.device(device)
        rank = dist.get_rank(group) if tp > 1 else 0
        if tp > 1 and dist.get_world_size(group) != tp:
            raise ValueError("tp must equal the size of the process group")
        self.cfg, self.max_seq, self.tp, self.batch = cfg, max_seq, tp, batch
        self.embed_tokens = nn.Embedding(cfg.vocab, cfg.hidden, device=device, dtype=torch.bfloat16)
        self.embed_tokens.weight.data = _rand_weight(cfg.vocab, cfg.hidden, seed + 7, device)
        self.layers = nn.ModuleList([Block(cfg, i, seed, device, tp, rank, group) for i in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden, cfg.eps)
        w = _rand_weight(cfg.vocab, cfg.hidden, seed + 11, device)
        piece = _vocab_piece(cfg.vocab, tp)
        self.lm_head = VocabShard(_linear_from(w[rank * piece:min((rank + 1) * piece, cfg.vocab)]), cfg.vocab, piece,
                                  group, tp)
        del w
        self.norm.to(device)
        for blk in self.layers:
            blk.input_layernorm.to(device)
            blk.post_attention_layernorm.to(device)
        self.cos, self.sin = _rope_tables(cfg.head_dim, max_seq, cfg.rope_theta, device)
        kvh = cfg.kv_heads // tp
        self.cache_k = torch.zeros(cfg.layers, batch, max_seq, kvh, cfg.head_dim, dtype=torch.bfloat16, device=device)
        self.cache_v = torch.zeros_like(self.cache_k)

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, pos0: torch.Tensor) -> torch.Tensor:
        """ids [batch, T] at positions pos0 .. pos0+T-1 (pos0: 0-d int64 device
        tensor); returns logits of the last position [batch, vocab]."""
        T = ids.shape[1]
        x = self.embed_tokens(ids)
        pos = pos0 + torch.arange(T, device=ids.device)
        keys = torch.arange(self.max_seq, device=ids.device)
        mask = (keys[None, :] <= pos[:, None])[None, None]              # [1, 1, T, S]
        if not x.is_cuda:
            cos, sin = self.cos[pos], self.sin[pos]
            for i, blk in enumerate(self.layers):
                x = blk(x, pos0, self.cache_k[i], self.cache_v[i], cos, sin, mask)
            h = self.norm(x[:, -1:, :])
            return self.lm_head(h).float().reshape(ids.shape[0], -1)
        # the GPU path: each residual add fused with the norm that follows it
        tables = (self.cos, self.sin)
        delta = None
        for i, blk in enumerate(self.layers):
            x, n1 = blk.input_layernorm.add_forward(x, delta)
            a = blk.self_attn(n1, pos0, self.cache_k[i], self.cache_v[i], None, None, mask, tables)
            x, n2 = blk.post_attention_layernorm.add_forward(x, a)
            delta = blk.mlp(n2)
        last = x[:, -1:, :].contiguous()
        _, h = self.norm.add_forward(last, delta[:, -1:, :].contiguous())
        return self.lm_head(h).float().reshape(ids.shape[0], -1)


class ResidentLinear(nn.Module):
    """A Linear whose weight is only the resident BF16X layout on the GPU:
    the fused GEMV for up to 16 rows of activations, the GEMM above."""

    def __init__(self, rw):
        super().__init__()
        self.rw = rw
        self.out_features, self.in_features = rw.rows, rw.in_f

    def forward(self, x):
        return self.rw.linear(x, None, out_dtype=torch.bfloat16)


@torch.no_grad()
def pack_model(model: LlamaModel) -> tuple[int, int]:
    """Replace every projection and lm_head by a ResidentLinear (packed on
    the GPU, the bf16 weight freed).  Returns (resident bytes, weights)."""
    from .opqk_linear import bf16x_quantize
    from .resident import ResidentWeight
    total = n = 0
    names = [(name, m) for name, m in model.named_modules() if isinstance(m, nn.Linear)]
    for name, m in names:
        dev = m.weight.device
        rw = ResidentWeight.from_packed(bf16x_quantize(m.weight.data, device=dev), device=dev)
        total += rw.nbytes()
        n += m.weight.numel()
        parent = model
        parts = name.split(".")
        for q in parts[:-1]:
            parent = getattr(parent, q)
        setattr(parent, parts[-1], ResidentLinear(rw))
        m.weight.data = torch.empty(0, device=dev)
    torch.cuda.empty_cache()
    return total, n


def use_peer_collectives(model: LlamaModel, peers) -> None:
    """After ``pack_model``: the o_proj / down_proj all-reduces and the
    lm_head all-gather of decode steps (up to 16 tokens per step) run inside
    the fused GEMVs over NVLink peer memory (``peers``: a PeerGroup over the
    model's tensor-parallel group, heap of ``peer_heap_bytes(model)``)."""
    if model.tp == 1:
        return
    for m in model.modules():
        if isinstance(m, (ColumnShard, VocabShard)):
            if not isinstance(m.lin, ResidentLinear):
                raise ValueError("use_peer_collectives needs a packed model (pack_model first)")
            m.attach_peers(peers, max(model.batch, 1))


def peer_heap_bytes(model: LlamaModel) -> int:
    """PeerGroup heap that use_peer_collectives carves for ``model``."""
    cfg, B, tp = model.cfg, max(model.batch, 1), model.tp
    per_layer = 2 * (tp * B * cfg.hidden * 8 + 256)
    return cfg.layers * per_layer + B * cfg.vocab * 8 + (1 << 20)


class GraphDecoder:
    """One decode step (a token in, the greedy next token out) captured as a
    CUDA graph and replayed; the position lives in a device tensor."""

    def __init__(self, model: LlamaModel, tok: torch.Tensor, pos: int):
        """tok [batch, 1]: the first tokens to feed, at position ``pos``.  The
        warm-up and capture write the cache row at ``pos`` only, which the
        first replay writes again."""
        self.model = model
        dev = model.cache_k.device
        self.tok = tok.reshape(-1, 1).clone()
        self.pos = torch.tensor(pos, dtype=torch.long, device=dev)
        self.next = torch.zeros_like(self.tok)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):                       # warm the kernels and the scratch on this stream
                self._step()
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._step()
        torch.cuda.current_stream(dev).wait_stream(s)

    def _step(self):
        logits = self.model(self.tok, self.pos)
        self.next.copy_(logits.argmax(-1, keepdim=True))

    def step(self):
        self.graph.replay()
        self.tok.copy_(self.next)
        self.pos += 1


@torch.no_grad()
def teacher_forced_logits(model: LlamaModel, prompt: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    """Logits [1 + n, batch, vocab] (fp32) of the prompt's last position and of
    n decode steps fed the given tokens [n, batch] (not the model's own
    choices), so two models -- bf16 and BF16X weights -- are compared on the
    same inputs at every step, without greedy divergence."""
    dev = prompt.device
    P = prompt.shape[1]
    out = [model(prompt, torch.zeros((), dtype=torch.long, device=dev)).float()]
    for i in range(tokens.shape[0]):
        pos = torch.tensor(P + i, dtype=torch.long, device=dev)
        out.append(model(tokens[i].reshape(-1, 1), pos).float())
    return torch.stack(out)


class fp32_linears:
    """Context manager: every plain nn.Linear of ``model`` computes in fp32
    (weights and activations upcast, product rounded back to the input
    dtype) instead of cuBLAS bf16.  Both are the exact-weight product and
    differ only in accumulation order and rounding, so the logits' distance
    between the two is the noise floor any exact-weight kernel is measured
    against."""

    def __init__(self, model: nn.Module):
        self.mods = [m for m in model.modules() if type(m) is nn.Linear]

    def __enter__(self):
        for m in self.mods:
            m.forward = (lambda x, m=m: F.linear(x.float(), m.weight.float(),
                                                 None if m.bias is None else m.bias.float()).to(x.dtype))
        return self

    def __exit__(self, *exc):
        for m in self.mods:
            del m.forward
        return False


def logits_rel_l2(a: torch.Tensor, b: torch.Tensor) -> tuple[float, float]:
    """(max, mean) over steps of ||a - b|| / ||b|| per step (fp64)."""
    d = (a.double() - b.double()).flatten(1).norm(dim=1) / b.double().flatten(1).norm(dim=1)
    return float(d.max()), float(d.mean())


@torch.no_grad()
def generate(model: LlamaModel, prompt: torch.Tensor, new_tokens: int, use_graph: bool = True):
    """Greedy generation: prefill ``prompt`` [batch, P], then ``new_tokens``
    decode steps.  Returns (tokens [new_tokens, batch], prefill ms, decode
    ms/token)."""
    dev = prompt.device
    P = prompt.shape[1]
    pos0 = torch.zeros((), dtype=torch.long, device=dev)
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    logits = model(prompt, pos0)
    b.record()
    torch.cuda.synchronize(dev)
    prefill_ms = a.elapsed_time(b)
    out = []
    if use_graph:
        dec = GraphDecoder(model, logits.argmax(-1, keepdim=True), P)
        a.record()
        for _ in range(new_tokens):
            out.append(dec.tok.clone())
            dec.step()
        b.record()
    else:
        tok = logits.argmax(-1, keepdim=True)
        pos = torch.tensor(P, dtype=torch.long, device=dev)
        a.record()
        for _ in range(new_tokens):
            out.append(tok)
            tok = model(tok, pos).argmax(-1, keepdim=True)
            pos = pos + 1
        b.record()
    torch.cuda.synchronize(dev)
    return torch.cat(out, dim=1).t().contiguous(), prefill_ms, a.elapsed_time(b) / max(new_tokens, 1)


__all__ = ["LlamaConfig", "CONFIGS", "LlamaModel", "ColumnShard", "VocabShard", "ResidentLinear", "pack_model",
           "GraphDecoder", "generate", "use_peer_collectives", "peer_heap_bytes", "teacher_forced_logits",
           "logits_rel_l2", "fp32_linears"]
