"""Torch dequantise-then-matmul backend for the model runner — TEST
INFRASTRUCTURE ONLY (the comparison arm of the greedy-identity test).

It restates, with plain torch ops on the GPU, the semantics of the reference's
extension operators that model_runner_v2 calls (src/ext/mxfp4_decode.cu,
mxfp4_linear.cu): activations quantised to MXFP4 with the quantize_expert_tensor
rules (quant/quantize_mxfp4.py:110-160), weights dequantised
(runtime/weight_store.py:27-44), products accumulated in fp32; the MoE block
as model_runner_v2 runs it (router lin_pq, softmax, top-8, renormalise,
gate/up, SwiGLU g / (1 + exp(-g)) * u in fp32, requantisation of h, down,
slot-ordered combine — runtime/model_runner_v2.py:183-208,
src/ext/mxfp4_decode.cu:252-299); attention with the reference attn_decode's
FP8 decoder (src/ext/mxfp4_decode.cu:362-421).  None of the library's kernels
run in it.  The router logits are summed in float64 (exact, as the library's
router computes them); everything else in fp32 through cuBLAS SGEMM.
"""

from __future__ import annotations

import torch

from oracle import attn as oa

_THRESH = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def quant_dequant(x: torch.Tensor) -> torch.Tensor:
    """Q(x) for fp32/bf16 rows: per 32-element block, scale 2^e with
    e = ceil(log2(max(amax / 6, 1e-30))) (code 127 / scale 1 for an all-zero
    block), magnitudes rounded to E2M1 with ties up; returned dequantised in
    fp32, columns padded to a multiple of 32 with zeros."""
    x = x.float()
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
    inv = torch.ldexp(torch.ones_like(t), -e)
    s = b * inv[..., None]
    mag = _MAG.to(x.device)[torch.bucketize(s.abs(), _THRESH.to(x.device), right=True)]
    v = torch.where(s < 0, -mag, mag)
    return (v * torch.ldexp(torch.ones_like(t), e)[..., None]).view(n, kp)


def dequant(wp: torch.Tensor, wsc: torch.Tensor) -> torch.Tensor:
    """Packed (N, Kp/2) + E8M0 (N, Kp/32) -> fp32 (N, Kp)."""
    n = wp.shape[0]
    kp = wp.shape[1] * 2
    codes = torch.empty((n, kp), dtype=torch.uint8, device=wp.device)
    codes[:, 0::2] = wp & 0xF
    codes[:, 1::2] = wp >> 4
    mag = _MAG.to(wp.device)[(codes & 7).long()]
    v = torch.where((codes & 8) != 0, -mag, mag).view(n, kp // 32, 32)
    return (v * torch.exp2(wsc.float() - 127.0)[..., None]).view(n, kp)


class TorchBackend:
    name = "torch dequantise-then-matmul"

    def __init__(self, model):
        torch.backends.cuda.matmul.allow_tf32 = False
        self.model = model
        self.cfg = model.cfg
        self._deq = {}
        self._lut = torch.from_numpy(oa.REF_DECODE).float().to(model.final_norm.device)

    def _w(self, w):
        key = w[0].data_ptr()
        d = self._deq.get(key)
        if d is None:
            d = self._deq[key] = dequant(w[0], w[1])
        return d

    def prequant(self, x):
        return quant_dequant(x), None

    def linear(self, xq, xsc, w, M, N, K):
        return torch.matmul(xq[:M], self._w(w).t())

    def moe_block(self, L, h):
        cfg = self.cfg
        mw = self.model.layers[L].moe
        a = quant_dequant(h)
        logits = (a.double() @ dequant(mw.router_wp, mw.router_sc).double().t()).float()
        probs = torch.softmax(logits, dim=-1)
        topv, topi = torch.topk(probs, cfg.top_k, dim=-1)
        topv = topv / topv.sum(-1, keepdim=True)
        T = h.shape[0]
        yd = torch.zeros((T, cfg.top_k, cfg.hidden), dtype=torch.float32, device=h.device)
        for e in torch.unique(topi).tolist():
            tok, slot = torch.where(topi == e)
            ae = a[tok]
            g = ae @ dequant(mw.gate_wp[e], mw.gate_sc[e]).t()
            u = ae @ dequant(mw.up_wp[e], mw.up_sc[e]).t()
            hh = g / (1.0 + torch.exp(-g)) * u
            yd[tok, slot] = quant_dequant(hh) @ dequant(mw.down_wp[e], mw.down_sc[e]).t()
        out = torch.zeros((T, cfg.hidden), dtype=torch.float32, device=h.device)
        for j in range(cfg.top_k):
            out = out + topv[:, j:j + 1] * yd[:, j]
        return out, topi.int()

    def attention(self, q, kvk, kvv, base, M):
        """The reference attn_decode semantics in fp32 torch: row m of each
        sequence attends to positions [0, base + m] of its cache."""
        B, _, Hq, D = q.shape
        Hkv = kvk.shape[2]
        S = base + M
        K = self._lut[kvk[:, :S].long()]                  # (B, S, Hkv, D)
        V = self._lut[kvv[:, :S].long()]
        K = K.repeat_interleave(Hq // Hkv, dim=2)         # (B, S, Hq, D)
        V = V.repeat_interleave(Hq // Hkv, dim=2)
        s = torch.einsum("bmhd,bshd->bhms", q.float(), K) / (D ** 0.5)
        pos = torch.arange(S, device=q.device)
        mask = pos[None, :] > (base + torch.arange(M, device=q.device))[:, None]
        s = s.masked_fill(mask[None, None], float("-inf"))
        p = torch.softmax(s, dim=-1)
        return torch.einsum("bhms,bshd->bmhd", p, V)
