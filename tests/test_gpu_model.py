"""BASELINE config 4 on one B200: the full random-init Qwen3-30B-A3B shape
(48 layers, 32 query / 4 KV heads, head_dim 128, vocab 151936, 128 experts,
top-8, MXFP4 experts and projections, FP8 KV cache), 1024-token synthetic
prompts (uniform random ids with a repeated 32-token motif), greedy decoding
of 128 steps at batch 1, 16 and 64, and the prompt-lookup speculative verify
(L = 4 drafts).

The same runner (moe_fused_inference_b200/model.py, the reference's
model_runner_v2 operation sequence) drives two backends: this library and a
torch dequantise-then-matmul restatement of the reference operators'
semantics (tests/torch_backend.py; its fp32 GEMMs of dequantised MXFP4
values are exact here — the same arm with float64 GEMMs is bit-identical).

What is asserted:
* the library against itself: speculative decoding (verify forwards of
  5 rows) emits exactly the greedy tokens (1-row forwards) — every kernel on
  the path computes a row the same way whatever the number of rows;
* the library against the torch arm on the prompt's forward pass: the
  residual stream agrees layer by layer (cosine >= 0.995) and the logits
  (cosine >= 0.99).
What is reported (printed): the first step at
which the two arms' greedy tokens differ and both arms' top-2 logit margins
there.  Exact identity over 128 steps is not attainable against an
independent arithmetic on this model: the library's softmax, attention and
tensor-core accumulation differ from the torch arm's by an ulp at times;
every MXFP4 requantisation of activations can turn that into a whole
quantisation step, and once a near-tied top-8 expert choice flips (about
layer 10 of the prompt's forward) the two hidden states separate.
"""

import json

import pytest
import torch

from moe_fused_inference_b200.model import (LibBackend, QwenConfig, Runner, SyntheticQwen,
                                            synthetic_prompts)
from tests.torch_backend import TorchBackend

pytestmark = pytest.mark.gpu

STEPS = 128
PROMPT = 1024


@pytest.fixture(scope="module")
def model():
    torch.manual_seed(0)
    return SyntheticQwen.build(QwenConfig(), seed=1)


@pytest.fixture(scope="module")
def backends(model):
    return LibBackend(model), TorchBackend(model)


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().flatten(), b.float().flatten(),
                                                 dim=0).item()


def test_prompt_forward_agrees_layer_by_layer(model, backends):
    lib, ref = backends
    prompt = synthetic_prompts(1, 64, model.cfg.vocab, seed=5)
    ta, tb = [], []
    la, _ = Runner(model, lib, 1, 128).forward(prompt, 0, trace=ta)
    lb, _ = Runner(model, ref, 1, 128).forward(prompt, 0, trace=tb)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    worst = min(_cos(xa, xb) for (_, _, xa), (_, _, xb) in zip(ta, tb))
    assert worst >= 0.995, worst
    assert _cos(la, lb) >= 0.99


@pytest.mark.parametrize("batch", [1, 16, 64])
def test_greedy_decode_against_reference_semantics(model, backends, batch):
    """The library decodes greedily (128 one-row steps per sequence); the
    torch arm then scores the same continuation teacher-forced (one batched
    pass over prompt + generated tokens), so every step compares the two
    arms' next-token choice on identical history.  Reported: the share of
    steps where they agree and the first disagreement with both margins."""
    lib, ref = backends
    prompt = synthetic_prompts(batch, PROMPT, model.cfg.vocab, seed=batch)
    max_len = PROMPT + STEPS + 8
    ta, ma = Runner(model, lib, batch, max_len).greedy(prompt, STEPS)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    assert bool(((ta >= 0) & (ta < model.cfg.vocab)).all())
    tb, mb = Runner(model, ref, batch, max_len).score(prompt, ta, chunk=128)
    same = ta == tb
    first = [int((~same[s]).nonzero()[0]) if not bool(same[s].all()) else STEPS
             for s in range(batch)]
    s0 = min(range(batch), key=lambda s: first[s])
    rep = {"batch": batch, "steps": STEPS, "agreeing_steps": float(same.float().mean()),
           "sequences_identical": sum(f == STEPS for f in first),
           "first_disagreement_step": first[s0]}
    if first[s0] < STEPS:
        t = first[s0]
        rep.update({"sequence": s0, "library_token": int(ta[s0, t]), "torch_token": int(tb[s0, t]),
                    "library_top2_margin": float(ma[s0, t]), "torch_top2_margin": float(mb[s0, t])})
    print("config4 greedy " + json.dumps(rep))
    # chance agreement over a 151,936-token vocabulary is nil; the arms pick
    # the same next token on about half of the steps of this random model,
    # whose top-2 logit margins are often below the arms' ~1e-1 logit spread
    assert rep["agreeing_steps"] >= 0.25


def test_speculative_decode_is_lossless(model, backends):
    """Prompt-lookup speculative decoding (runtime/spec_decoder.py:22-122) on
    the library: verify forwards of 1 + 4 rows (attn_decode with M = 5, the
    batched projections and MoE) must reproduce the plain greedy tokens bit
    for bit.  The prompt's motif makes the lookup propose drafts, so verify
    forwards with several rows do run; how many drafts a random-init model
    accepts is luck (0 to a few), so only the proposals are asserted."""
    lib, _ = backends
    prompt = synthetic_prompts(1, PROMPT, model.cfg.vocab, seed=101)
    max_len = PROMPT + STEPS + 16
    greedy, _ = Runner(model, lib, 1, max_len).greedy(prompt, STEPS)
    r = Runner(model, lib, 1, max_len)
    spec, forwards, accepted = r.speculative(prompt, STEPS)
    print(f"config4 speculative: {STEPS} tokens in {forwards} verify forwards, "
          f"{r.spec_stats['drafted']} drafted tokens proposed, {accepted} accepted")
    assert torch.equal(spec.to(greedy.device), greedy[0])
    assert r.spec_stats["drafted"] > 0


@pytest.mark.parametrize("batch", [1, 16])
def test_graph_decode_matches_eager_greedy(model, backends, batch):
    """Config 4's decode as one captured CUDA graph per step (the device-
    routed MoE layer leaves nothing on the step for the host; the reference's
    graph attempt failed on its routing .tolist()): the replayed steps emit
    exactly the eager greedy tokens."""
    from moe_fused_inference_b200.model import GraphDecoder
    lib, _ = backends
    steps = 24
    prompt = synthetic_prompts(batch, 256, model.cfg.vocab, seed=31)
    max_len = 256 + steps + 8
    greedy, _ = Runner(model, lib, batch, max_len).greedy(prompt, steps)
    gd = GraphDecoder(Runner(model, lib, batch, max_len), steps)
    gd.start(prompt)
    toks = gd.decode(steps)
    torch.cuda.synchronize()
    assert torch.equal(toks, greedy)
