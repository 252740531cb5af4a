"""The end-to-end decoder with BF16X linears (every projection and lm_head):
prefill logits against the same model with bf16 weights, and CUDA-graph
decode against eager decode."""
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200.llama_e2e import CONFIGS, LlamaModel, generate, pack_model
from tests.gpu_util import rel_l2

pytestmark = pytest.mark.gpu


def test_packed_model_matches_bf16_and_graph_decode():
    dev = torch.device("cuda", 0)
    cfg = CONFIGS["tiny"]
    prompt = torch.randint(0, cfg.vocab, (1, 40), generator=torch.Generator().manual_seed(1)).to(dev)
    model = LlamaModel(cfg, 64, dev, seed=3)
    pos0 = torch.zeros((), dtype=torch.long, device=dev)
    ref = model(prompt, pos0).cpu().numpy()
    total, n = pack_model(model)
    per_layer = (cfg.hidden * (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim + cfg.heads * cfg.head_dim * cfg.hidden
                 + 3 * cfg.hidden * cfg.ffn)
    assert n == cfg.layers * per_layer + cfg.hidden * cfg.vocab
    assert total < 2 * n                                     # fewer bytes than bf16
    got = model(prompt, pos0).cpu().numpy()
    assert rel_l2(got, ref) < 2e-2                            # bf16 activations in both
    tok_graph, _, _ = generate(model, prompt, 12, use_graph=True)
    tok_eager, _, _ = generate(model, prompt, 12, use_graph=False)
    assert torch.equal(tok_graph, tok_eager)
    _lib.check_device_status()
