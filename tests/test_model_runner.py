"""The model runner's plumbing on CPU (moe_fused_inference_b200/model.py):
a tiny synthetic model quantised with the oracle, driven by the torch
backend (tests/torch_backend.py) — prefill in chunks, greedy decode of a
batch, and the prompt-lookup speculative decode, which is lossless: it must
emit the greedy tokens."""

import numpy as np
import torch

from moe_fused_inference_b200.layer import MoELayerWeights
from moe_fused_inference_b200.model import QwenConfig, Runner, SyntheticQwen, synthetic_prompts
from oracle import mxfp4 as mx
from tests.torch_backend import TorchBackend


def _tiny_model(seed=0):
    cfg = QwenConfig(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=32, vocab=97, experts=8,
                     top_k=2, inter=32)
    rng = np.random.default_rng(seed)

    def packed(n, k):
        p, c = mx.quantize_rows(mx.bf16_round(rng.standard_normal((n, k)).astype(np.float32) * 0.2))
        return torch.from_numpy(p), torch.from_numpy(c)

    def norm(n):
        return torch.from_numpy(1.0 + 0.02 * rng.standard_normal(n).astype(np.float32)).bfloat16()

    H, D = cfg.hidden, cfg.head_dim
    m = SyntheticQwen(cfg, packed(cfg.vocab, H), packed(cfg.vocab, H), norm(H))
    from moe_fused_inference_b200.model import LayerWeights
    for _ in range(cfg.layers):
        W = mx.make_layer(rng, n_experts=cfg.experts, hidden=H, inter=cfg.inter, std=0.2)
        t = torch.from_numpy
        moe = MoELayerWeights(t(W.wg), t(W.sg), t(W.wu), t(W.su), t(W.wd), t(W.sd), t(W.wr), t(W.sr))
        m.layers.append(LayerWeights(packed(cfg.heads * D, H), packed(cfg.kv_heads * D, H),
                                     packed(cfg.kv_heads * D, H), packed(H, cfg.heads * D),
                                     norm(D), norm(D), norm(H), norm(H), moe))
    return m


def test_runner_greedy_and_speculative_on_cpu():
    m = _tiny_model()
    be = TorchBackend(m)
    prompt = synthetic_prompts(2, 80, m.cfg.vocab, seed=3, motif=8, device="cpu")
    toks, margins = Runner(m, be, 2, 128).greedy(prompt, 12)
    assert toks.shape == (2, 12) and margins.shape == (2, 12)
    assert bool((margins >= 0).all())
    # the prompt's chunking does not change the result
    toks2, _ = Runner(m, be, 2, 128).greedy(prompt, 12, chunk=16)
    assert torch.equal(toks, toks2)
    r = Runner(m, be, 1, 128)
    spec, forwards, accepted = r.speculative(prompt[:1], 12, n_gram=3)
    assert torch.equal(spec, toks[0])
    assert forwards <= 12
    # teacher-forced scoring of the greedy continuation reproduces it
    am, mg = Runner(m, be, 2, 128).score(prompt, toks, chunk=5)
    assert torch.equal(am, toks) and mg.shape == toks.shape
