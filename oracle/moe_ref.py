"""CPU port of the reference's dequantise-then-matmul MoE layer — TEST / BASELINE ONLY.

Restates, in torch on the host CPU, the reference's v1 MoE path that
BASELINE config 1 names:
  * router: ``ModelRunner.moe_route`` (runtime/model_runner.py:99-108):
    logits = F.linear(h, Wr) in the activation dtype, softmax in float32,
    top-k, renormalise, cast scores back to the activation dtype;
  * experts: ``ModelRunner.moe_compute(variant="mxfp4")``
    (runtime/model_runner.py:110-132): per active expert, gather its tokens,
    silu(x Wg^T) * (x Wu^T), then (.) Wd^T, all bf16 F.linear on weights
    dequantised once with ``mxfp4_reconstruct_gpu`` semantics
    (runtime/weight_store.py:27-44, cast to bf16 at :262), and
    ``index_add_`` of the score-weighted rows.

Used by ``bench.py`` (cpu_baseline and --impl reference) and by tests that pin
it against ``tests/golden/route_moe.npz`` (generated from the reference
itself).  Nothing in the CUDA product path imports it.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import mxfp4 as mx


_THRESH = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=torch.float32)
_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)


def quant_dequant_bf16(w: torch.Tensor) -> torch.Tensor:
    """Quantise (N, K) CPU weights to MXFP4 and reconstruct them as bf16 —
    quantize_expert_tensor (quant/quantize_mxfp4.py:110-160) followed by
    mxfp4_reconstruct_gpu(...).to(bf16) (runtime/weight_store.py:27-44,262),
    vectorised with multi-threaded torch CPU ops so a 128-expert layer takes
    seconds.  Equal to dequantize_rows(*quantize_rows(w)) (checked by
    tests/test_oracle_golden.py)."""
    x = w.to(torch.float32)
    n, k = x.shape
    kp = (k + 31) // 32 * 32
    if kp != k:
        x = torch.nn.functional.pad(x, (0, kp - k))
    b = x.view(n, kp // 32, 32)
    amax = b.abs().amax(-1)
    t = torch.clamp(amax / 6.0, min=1e-30)
    m, e = torch.frexp(t)
    e = torch.where(m == 0.5, e - 1, e)
    e = torch.where(amax > 0, e, torch.zeros_like(e))
    scale = torch.ldexp(torch.ones_like(t), e)
    s = b / scale[..., None]
    mag = torch.bucketize(s.abs(), _THRESH, right=True)
    v = _MAG[mag]
    v = torch.where(s < 0, -v, v)
    out = (v * scale[..., None]).view(n, kp)[:, :k]
    return out.to(torch.bfloat16)


def dequant_bf16(packed: np.ndarray, codes: np.ndarray, k: int) -> torch.Tensor:
    """packed MXFP4 -> bf16 tensor (reference runtime/weight_store.py:27-44,262)."""
    return torch.from_numpy(mx.dequantize_rows(packed, codes, k)).to(torch.bfloat16)


class CpuMoELayer:
    """A MoE layer with experts dequantised to bf16 up front (excluded from timing,
    as the reference's LRU cache holds dequantised experts)."""

    def __init__(self, W: "mx.MoELayerWeights", router_bf16: torch.Tensor | None = None,
                 top_k: int = 8, norm_topk_prob: bool = True, experts=None):
        self.top_k = top_k
        self.norm = norm_topk_prob
        hidden = W.wg.shape[2] * 2
        inter = W.wg.shape[1]
        if router_bf16 is None:
            router_bf16 = dequant_bf16(W.wr, W.sr, hidden)
        self.wr = router_bf16
        ids = range(W.n_experts) if experts is None else experts
        self.experts = {}
        for e in ids:
            self.experts[e] = (
                dequant_bf16(W.wg[e], W.sg[e], hidden),
                dequant_bf16(W.wu[e], W.su[e], hidden),
                dequant_bf16(W.wd[e], W.sd[e], inter),
            )

    def route(self, h: torch.Tensor):
        logits = F.linear(h, self.wr)
        probs = F.softmax(logits.float(), dim=-1)
        topv, topi = torch.topk(probs, self.top_k, dim=-1)
        if self.norm:
            topv = topv / topv.sum(dim=-1, keepdim=True)
        return logits, topi, topv.to(logits.dtype)

    def compute(self, h: torch.Tensor, topi: torch.Tensor, scores: torch.Tensor):
        out = torch.zeros_like(h)
        for e, (wg, wu, wd) in self.experts.items():
            idx, slots = torch.where(topi == e)
            if idx.numel() == 0:
                continue
            xt = h[idx]
            hh = F.silu(F.linear(xt, wg)) * F.linear(xt, wu)
            y = F.linear(hh, wd)
            out.index_add_(0, idx, y * scores[idx, slots].unsqueeze(-1))
        return out

    @staticmethod
    def from_bf16(wg, wu, wd, wr, top_k=8, norm_topk_prob=True):
        """Build from lists of bf16 expert weights (already dequantised) and a
        bf16 router, skipping the packed form."""
        obj = CpuMoELayer.__new__(CpuMoELayer)
        obj.top_k, obj.norm, obj.wr = top_k, norm_topk_prob, wr
        obj.experts = {e: (wg[e], wu[e], wd[e]) for e in range(len(wg))}
        return obj

    def forward(self, h: torch.Tensor):
        logits, topi, scores = self.route(h)
        return self.compute(h, topi, scores), topi, scores, logits
