"""The 1B-class decoder (hidden 2048, 24 layers, GQA 16/8, SwiGLU 6144, vocab
73448) at its real size: logits with every projection and lm_head
BF16X-packed against the same model with bf16 weights, on the prompt and on
teacher-forced decode steps (the same tokens fed to both, so greedy
divergence between nearly tied random-init logits does not enter).  The
decode is bit-exact, so what differs is only the fp32 accumulation order of
the fused kernels against cuBLAS and the bf16 rounding of each layer's
output, compounded over 24 layers.  The noise floor of that is measured on
the same inputs: the same bf16 weights with every linear computed as an fp32
GEMM instead of cuBLAS bf16.  Tolerance: the packed model within 1.5x that
floor of the cuBLAS bf16 run (relative L2 of the logits, per step), and
under 5e-2 absolute."""
import pytest
import torch

from bfloat16x_b200 import _lib
from bfloat16x_b200.llama_e2e import (CONFIGS, LlamaModel, fp32_linears, generate, logits_rel_l2, pack_model,
                                      teacher_forced_logits)

pytestmark = pytest.mark.gpu
TOL_FLOOR = 1.5
TOL_ABS = 5e-2


def test_1b_logits_packed_vs_bf16():
    dev = torch.device("cuda", 0)
    cfg = CONFIGS["1b"]
    prompt = torch.randint(0, cfg.vocab, (1, 128), generator=torch.Generator().manual_seed(3)).to(dev)
    model = LlamaModel(cfg, 160, dev, seed=0)
    tok, _, _ = generate(model, prompt, 8, use_graph=False)
    ref = teacher_forced_logits(model, prompt, tok)
    with fp32_linears(model):
        alt = teacher_forced_logits(model, prompt, tok)
    floor_max, floor_mean = logits_rel_l2(alt, ref)
    pack_model(model)
    got = teacher_forced_logits(model, prompt, tok)
    mx, mean = logits_rel_l2(got, ref)
    assert mx < TOL_ABS and mx <= TOL_FLOOR * floor_max and mean <= TOL_FLOOR * floor_mean, \
        (mx, mean, floor_max, floor_mean)
    # the CUDA-graph decode of the packed model takes the same steps as its eager decode
    tg, _, _ = generate(model, prompt, 8, use_graph=True)
    te, _, _ = generate(model, prompt, 8, use_graph=False)
    assert torch.equal(tg, te)
    _lib.check_device_status()
    del model
    torch.cuda.empty_cache()
