"""End-to-end decoder for the BF16X path: a Llama-style model whose linear
layers (attention and MLP projections and lm_head) are BF16X-packed and run
through the fused decode+GEMV (one token) and decode+GEMM (prefill) kernels.

It exists to measure the hot path inside a model: ms per generated token
against the same model with plain bf16 weights (cuBLAS), at batch 1 after a
prompt prefill, for the two decoder configurations of the benchmark
(``CONFIGS``).  Weights are random N(0, 0.02) (no checkpoints); attention
uses torch's scaled_dot_product_attention over a static KV cache, so one
decode step has static shapes and is replayed as a CUDA graph.

"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


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
    # 1B-class Llama-style decoder
    "1b": LlamaConfig(hidden=2048, layers=24, heads=16, kv_heads=8, head_dim=128, ffn=6144, vocab=73448),
    # 8B Llama-3-style decoder
    "8b": LlamaConfig(hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256),
    # a small one for tests
    "tiny": LlamaConfig(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000),
}


class RMSNorm(nn.Module):
    def __init__(self, n: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n, dtype=torch.bfloat16), requires_grad=False)
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (y * self.weight.float()).to(x.dtype)


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


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig, tp: int = 1):
        super().__init__()
        self.cfg, self.tp = cfg, tp
        self.h, self.kvh, self.d = cfg.heads // tp, cfg.kv_heads // tp, cfg.head_dim
        # q, k and v projections as one [q; k; v] weight: one GEMV per step
        self.qkv_proj = nn.Linear(cfg.hidden, (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim, bias=False)
        self.o_proj = nn.Linear(cfg.heads * cfg.head_dim, cfg.hidden, bias=False)

    def forward(self, x, pos0, cache_k, cache_v, cos, sin, mask):
        B, T, _ = x.shape
        qkv = self.qkv_proj(x)
        nq, nk = self.h * self.d, self.kvh * self.d
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
    def __init__(self, cfg: LlamaConfig, tp: int = 1):
        super().__init__()
        # gate and up projections as one [gate; up] weight
        self.ffn = cfg.ffn
        self.gate_up_proj = nn.Linear(cfg.hidden, 2 * cfg.ffn, bias=False)
        self.down_proj = nn.Linear(cfg.ffn, cfg.hidden, bias=False)

    def forward(self, x):
        gu = self.gate_up_proj(x)
        return self.down_proj(F.silu(gu[..., :self.ffn]) * gu[..., self.ffn:])


class Block(nn.Module):
    def __init__(self, cfg: LlamaConfig, tp: int = 1):
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.eps)
        self.self_attn = Attention(cfg, tp)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.eps)
        self.mlp = MLP(cfg, tp)

    def forward(self, x, pos0, ck, cv, cos, sin, mask):
        x = x + self.self_attn(self.input_layernorm(x), pos0, ck, cv, cos, sin, mask)
        return x + self.mlp(self.post_attention_layernorm(x))


class LlamaModel(nn.Module):
    """Llama-style decoder with a static KV cache of ``max_seq`` positions."""

    def __init__(self, cfg: LlamaConfig, max_seq: int, device, seed: int = 0, tp: int = 1):
        super().__init__()
        if tp != 1:
            raise NotImplementedError("the end-to-end decoder runs on one GPU")
        self.cfg, self.max_seq, self.tp = cfg, max_seq, tp
        self.embed_tokens = nn.Embedding(cfg.vocab, cfg.hidden)
        self.layers = nn.ModuleList([Block(cfg, tp) for _ in range(cfg.layers)])
        self.norm = RMSNorm(cfg.hidden, cfg.eps)
        self.lm_head = nn.Linear(cfg.hidden, cfg.vocab, bias=False)
        self.to(device=device, dtype=torch.bfloat16)
        gd = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for p in self.parameters():
                if p.dim() == 2:
                    p.normal_(0.0, 0.02, generator=gd)
        self.cos, self.sin = _rope_tables(cfg.head_dim, max_seq, cfg.rope_theta, device)
        kvh = cfg.kv_heads // tp
        self.cache_k = torch.zeros(cfg.layers, 1, max_seq, kvh, cfg.head_dim, dtype=torch.bfloat16, device=device)
        self.cache_v = torch.zeros_like(self.cache_k)

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, pos0: torch.Tensor) -> torch.Tensor:
        """ids [1, T] at positions pos0 .. pos0+T-1 (pos0: 0-d int64 device
        tensor); returns logits of the last position [1, vocab]."""
        T = ids.shape[1]
        x = self.embed_tokens(ids)
        pos = pos0 + torch.arange(T, device=ids.device)
        cos, sin = self.cos[pos], self.sin[pos]
        keys = torch.arange(self.max_seq, device=ids.device)
        mask = (keys[None, :] <= pos[:, None])[None, None]              # [1, 1, T, S]
        for i, blk in enumerate(self.layers):
            x = blk(x, pos0, self.cache_k[i], self.cache_v[i], cos, sin, mask)
        h = self.norm(x[:, -1:, :])
        return self.lm_head(h).float().reshape(1, -1)


class ResidentLinear(nn.Module):
    """A Linear whose weight is only the resident BF16X layout on the GPU:
    the fused GEMV for up to 8 rows of activations, the GEMM above."""

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


class GraphDecoder:
    """One decode step (a token in, the greedy next token out) captured as a
    CUDA graph and replayed; the position lives in a device tensor."""

    def __init__(self, model: LlamaModel, tok: torch.Tensor, pos: int):
        """tok [1, 1]: the first token to feed, at position ``pos``.  The
        warm-up and capture write the cache row at ``pos`` only, which the
        first replay writes again."""
        self.model = model
        dev = model.cache_k.device
        self.tok = tok.reshape(1, 1).clone()
        self.pos = torch.tensor(pos, dtype=torch.long, device=dev)
        self.next = torch.zeros(1, 1, dtype=torch.long, device=dev)
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
def generate(model: LlamaModel, prompt: torch.Tensor, new_tokens: int, use_graph: bool = True):
    """Greedy generation: prefill ``prompt`` [1, P], then ``new_tokens``
    decode steps.  Returns (tokens [new_tokens], prefill ms, decode ms/token)."""
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
    return torch.cat(out).reshape(-1), prefill_ms, a.elapsed_time(b) / max(new_tokens, 1)


__all__ = ["LlamaConfig", "CONFIGS", "LlamaModel", "ResidentLinear", "pack_model", "GraphDecoder", "generate"]
