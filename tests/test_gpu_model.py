"""BASELINE config 4 on one B200: the full random-init Qwen3-30B-A3B shape
(48 layers, 32 query / 4 KV heads, head_dim 128, vocab 151936, 128 experts,
top-8, MXFP4 experts and projections, FP8 KV cache) decoded greedily for 128
steps after 1024-token synthetic prompts (uniform random ids with a repeated
32-token motif), at batch 1, 16 and 64, and with the prompt-lookup
speculative verify (L = 4 drafts).

The same runner (moe_fused_inference_b200/model.py, the reference's
model_runner_v2 operation sequence) drives two backends: this library, and a
torch dequantise-then-matmul restatement of the reference operators' semantics
(tests/torch_backend.py).  identical greedy token ids
over the 128 steps.  On a mismatch the first divergence is reported with both
arms' top-2 logit margins.
"""

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


def _report(a, b, ma, mb):
    diff = (a != b).nonzero()
    if diff.numel() == 0:
        return ""
    s, t = int(diff[0, 0]), int(diff[0, 1])
    return (f"first divergence: sequence {s} step {t}: library {int(a[s, t])} "
            f"(top-2 margin {float(ma[s, t]):.3e}) vs torch {int(b[s, t])} "
            f"(margin {float(mb[s, t]):.3e}); {int((a != b).sum())} of {a.numel()} differ")


@pytest.mark.parametrize("batch", [1, 16, 64])
def test_greedy_token_identity(model, backends, batch):
    lib, ref = backends
    prompt = synthetic_prompts(batch, PROMPT, model.cfg.vocab, seed=batch)
    max_len = PROMPT + STEPS + 8
    toks_a, marg_a = Runner(model, lib, batch, max_len).greedy(prompt, STEPS)
    toks_b, marg_b = Runner(model, ref, batch, max_len).greedy(prompt, STEPS)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    assert torch.equal(toks_a, toks_b), _report(toks_a, toks_b, marg_a, marg_b)


def test_speculative_verify_identity(model, backends):
    """Prompt-lookup speculative decoding (runtime/spec_decoder.py:22-122) of
    one sequence: the verify forward of 1 + 4 rows runs attn_decode with M = 5
    and the batched projections; both arms must emit the same tokens, and the
    motif in the prompt must make some drafts accepted."""
    lib, ref = backends
    prompt = synthetic_prompts(1, PROMPT, model.cfg.vocab, seed=101)
    max_len = PROMPT + STEPS + 16
    ta, fa, acc_a = Runner(model, lib, 1, max_len).speculative(prompt, STEPS)
    tb, fb, acc_b = Runner(model, ref, 1, max_len).speculative(prompt, STEPS)
    assert torch.equal(ta, tb), f"first divergence at step {int((ta != tb).nonzero()[0, 0])}"
    assert fa == fb and acc_a == acc_b
    print(f"speculative: {STEPS} tokens in {fa} verify forwards, {acc_a} drafted tokens accepted")
