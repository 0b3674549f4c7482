"""The reference runners' MoE call sequences through the drop-in operators.

The reference's runner code cannot run here (its tree is not on the GPU
boxes and its own kernels are sm_120a-only), so these tests restate, step for
step, the two places it calls the operators, with this library's fp4_ext in
the place of the reference's extension:

* runtime/model_runner_v2.py:183-208 (decode MoE block of forward_decode):
  prequant -> lin_pq router -> softmax, top-8, renormalise -> .tolist() ->
  Python pointer lists -> moe_gateup -> moe_down -> moe_combine;
* runtime/model_runner.py:99-132 (moe_route + moe_compute, variant
  "mxfp4_mma"): F.linear router on the bf16 gate weight, softmax / top-k /
  renormalise, scores in the logits' dtype, then per expert
  get_ext().forward for gate and up, silu(g) * u in torch, forward for down,
  y in the activation dtype, index_add_ of y * score.

Every GEMM is checked against the float64 oracle of the same quantised
operands (max relative error 1e-4), the rest of the chain against the
oracle's restatement of the same host steps.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from moe_fused_inference_b200 import fp4_ext
from oracle import mxfp4 as mx
from tests.conftest import cosine, max_rel_err

pytestmark = pytest.mark.gpu

E_ALL, H, MI, K = 16, 2048, 768, 8


def _experts(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dext = fp4_ext.get_decode_ext()
    ex = []
    for _ in range(E_ALL):
        mats = {}
        for name, (n, k) in (("gate", (MI, H)), ("up", (MI, H)), ("down", (H, MI))):
            w = (torch.randn((n, k), generator=g, device="cuda") * 0.02).bfloat16()
            wp, wsc = dext.prequant(w)
            mats[name] = {"wp": wp, "wsc": wsc}
        ex.append(mats)
    router = (torch.randn((E_ALL, H), generator=g, device="cuda") * 0.02).bfloat16()
    return ex, router


def _np(t):
    return t.detach().cpu().numpy()


def test_v2_decode_moe_block_sequence():
    """runtime/model_runner_v2.py:183-208 for one token."""
    ex, router = _experts(11)
    dext = fp4_ext.get_decode_ext()
    rwp, rws = dext.prequant(router)
    g = torch.Generator(device="cuda").manual_seed(5)
    hp2 = torch.randn((1, H), generator=g, device="cuda").bfloat16()
    hp2q, hp2s = dext.prequant(hp2.contiguous())
    gate_logits = dext.lin_pq(hp2q, hp2s, rwp, rws, 1, E_ALL, H)
    router_probs = F.softmax(gate_logits, dim=-1)
    topv, topi = torch.topk(router_probs, K, dim=-1)
    topv = topv / topv.sum(dim=-1, keepdim=True)
    ids = topi.view(-1).tolist()
    gwp = [ex[e]["gate"]["wp"] for e in ids]
    gsc = [ex[e]["gate"]["wsc"] for e in ids]
    uwp = [ex[e]["up"]["wp"] for e in ids]
    usc = [ex[e]["up"]["wsc"] for e in ids]
    dwp = [ex[e]["down"]["wp"] for e in ids]
    dsc = [ex[e]["down"]["wsc"] for e in ids]
    gu = dext.moe_gateup(hp2q, hp2s, gwp + uwp, gsc + usc, K, 1, MI, H)
    yd = dext.moe_down(gu, dwp, dsc, K, 1, H, MI)
    moe = dext.moe_combine(yd, topv.view(1, K).float(), 1)[0]
    torch.cuda.synchronize()
    assert moe.shape == (H,) and moe.dtype == torch.float32

    # oracle: the router logits, then each slot's chain from the same operands
    xq, xs = _np(hp2q), _np(hp2s)
    lg = mx.mx_gemm_f64(xq, xs, _np(rwp), _np(rws))[0]
    assert max_rel_err(_np(gate_logits)[0], lg) <= 1e-4
    gu_n, yd_n = _np(gu), _np(yd)
    for s, e in enumerate(ids):
        rg = mx.mx_gemm_f64(xq, xs, _np(ex[e]["gate"]["wp"]), _np(ex[e]["gate"]["wsc"]))[0]
        ru = mx.mx_gemm_f64(xq, xs, _np(ex[e]["up"]["wp"]), _np(ex[e]["up"]["wsc"]))[0]
        assert max_rel_err(gu_n[s, :MI], rg) <= 1e-4
        assert max_rel_err(gu_n[s, MI:], ru) <= 1e-4
        hq, hs = mx.quantize_rows(mx.silu_mul(gu_n[s:s + 1, :MI], gu_n[s:s + 1, MI:]))
        rd = mx.mx_gemm_f64(hq, hs, _np(ex[e]["down"]["wp"]), _np(ex[e]["down"]["wsc"]))[0]
        assert max_rel_err(yd_n[s], rd) <= 1e-4
    assert np.array_equal(_np(moe), mx.combine(yd_n, _np(topv.float()), 1)[0])


def test_v1_mxfp4_mma_moe_compute_sequence():
    """runtime/model_runner.py:99-132 (moe_route, moe_compute variant
    "mxfp4_mma") for 5 tokens over 16 experts."""
    ex, router = _experts(12)
    ext = fp4_ext.get_ext()
    T = 5
    g = torch.Generator(device="cuda").manual_seed(6)
    h = torch.randn((T, H), generator=g, device="cuda").bfloat16()
    # moe_route
    logits = F.linear(h, router)
    router_probs = F.softmax(logits.float(), dim=-1)
    topv, topi = torch.topk(router_probs, K, dim=-1)
    topv = topv / topv.sum(dim=-1, keepdim=True)
    scores = topv.to(logits.dtype)
    # moe_compute("mxfp4_mma")
    out = torch.zeros_like(h)
    ref = np.zeros((T, H), np.float64)
    for e in range(E_ALL):
        idx, slots = torch.where(topi == e)
        if idx.numel() == 0:
            continue
        xt = h[idx]
        wg, wu, wd = ex[e]["gate"], ex[e]["up"], ex[e]["down"]
        gg = ext.forward(xt, wg["wp"], wg["wsc"])
        uu = ext.forward(xt, wu["wp"], wu["wsc"])
        hh = F.silu(gg) * uu
        y = ext.forward(hh, wd["wp"], wd["wsc"])
        y = y.to(out.dtype)
        out.index_add_(0, idx, y * scores[idx, slots].unsqueeze(-1))
        torch.cuda.synchronize()
        # each forward against the float64 oracle of its own quantised input
        # (the binding casts bf16 and fp32 inputs to fp16 first)
        xq, xs = mx.quantize_rows(_np(xt.half().float()))
        assert max_rel_err(_np(gg), mx.mx_gemm_f64(xq, xs, _np(wg["wp"]), _np(wg["wsc"]))) <= 1e-4
        assert max_rel_err(_np(uu), mx.mx_gemm_f64(xq, xs, _np(wu["wp"]), _np(wu["wsc"]))) <= 1e-4
        hq, hs = mx.quantize_rows(_np(hh.half().float()))
        yr = mx.mx_gemm_f64(hq, hs, _np(wd["wp"]), _np(wd["wsc"]))
        assert max_rel_err(_np(y.float()), yr) <= 1e-2  # y rounded to bf16
        w = _np(scores[idx, slots].float())
        for i, t in enumerate(_np(idx)):
            ref[t] += w[i] * yr[i]
    torch.cuda.synchronize()
    # the runner accumulates in bf16 (index_add_ on a bf16 tensor)
    got = _np(out.float())
    assert max_rel_err(got, ref) <= 2e-2
    assert cosine(got, ref) >= 0.999
