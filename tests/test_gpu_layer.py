"""Fused device-routed MoE layer (MoELayer / mfi_moe_layer) vs the kernel-path oracle.

Contract: top-k indices and router logits bit-exact;
layer output max relative error <= 1e-2 and cosine >= 0.999 versus the
fp32-accumulated dequantised reference (the oracle accumulates in float64).
"""

import numpy as np
import pytest
import torch

from moe_fused_inference_b200.layer import MoELayer, MoELayerWeights, random_layer_weights
from oracle import mxfp4 as mx
from tests.conftest import cosine, max_rel_err

pytestmark = pytest.mark.gpu


def oracle_weights(w: MoELayerWeights):
    c = lambda t: t.cpu().numpy()
    return mx.MoELayerWeights(c(w.gate_wp), c(w.gate_sc), c(w.up_wp), c(w.up_sc),
                              c(w.down_wp), c(w.down_sc), c(w.router_wp), c(w.router_sc))


@pytest.fixture(scope="module")
def qwen_layer():
    return random_layer_weights(n_experts=128, hidden=2048, inter=768, std=0.02, seed=1)


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_layer_decode_sizes(qwen_layer, T):
    layer = MoELayer(qwen_layer, top_k=8)
    g = torch.Generator(device="cuda").manual_seed(100 + T)
    x = torch.randn((T, 2048), generator=g, device="cuda").bfloat16()
    logits = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    out, topi, topw = layer(x, logits=logits)
    ref = mx.moe_layer(x.float().cpu().numpy(), oracle_weights(qwen_layer), topk=8)
    assert np.array_equal(logits.cpu().numpy(), ref["logits"]), "router logits must be bit-exact"
    assert np.array_equal(topi.cpu().numpy(), ref["idx"]), "top-k indices must be bit-exact"
    np.testing.assert_allclose(topw.cpu().numpy(), ref["w"], rtol=2e-6, atol=1e-7)
    o = out.cpu().numpy()
    assert cosine(o, ref["out"]) >= 0.999
    assert max_rel_err(o, ref["out"]) <= 1e-2


def test_layer_small_odd_config():
    """E = 16 experts, top-4, hidden 256, inter 96 (3 blocks), T = 13."""
    w = random_layer_weights(n_experts=16, hidden=256, inter=96, std=0.05, seed=4)
    layer = MoELayer(w, top_k=4)
    x = torch.randn((13, 256), device="cuda").bfloat16()
    out, topi, topw = layer(x)
    ref = mx.moe_layer(x.float().cpu().numpy(), oracle_weights(w), topk=4)
    assert np.array_equal(topi.cpu().numpy(), ref["idx"])
    assert cosine(out.cpu().numpy(), ref["out"]) >= 0.999
    assert max_rel_err(out.cpu().numpy(), ref["out"]) <= 1e-2


def test_layer_repeatable_and_graph_capturable(qwen_layer):
    layer = MoELayer(qwen_layer, top_k=8)
    x = torch.randn((8, 2048), device="cuda").bfloat16()
    out1, ti1, tw1 = layer(x)
    out2, ti2, tw2 = layer(x)
    assert torch.equal(out1, out2) and torch.equal(ti1, ti2) and torch.equal(tw1, tw2)
    o = torch.empty_like(out1)
    ti = torch.empty_like(ti1)
    tw = torch.empty_like(tw1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer(x, out=o, topi=ti, topw=tw)  # warm the workspace outside capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer(x, out=o, topi=ti, topw=tw)
    o.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(o, out1)


@pytest.mark.parametrize("T,path", [(1, "decode"), (8, "decode"), (64, "decode"),
                                    (600, "prefill"), (300, "prefill")])
def test_layer_fused_rms_norm(qwen_layer, T, path):
    """RMSNorm fused into the router (the MoE block's post-attention
    layernorm, runtime/model_runner.py:20-25 at runtime/model_runner_v2.py:183):
    the layer takes the residual stream; its routing must equal the oracle's
    on rms_norm_bf16(x) bit for bit and its output meet the layer contract.
    Covers the decode cluster router (T <= 64), the tensor-core prefill router
    (T = 600) and the cluster router with the prefill's count-based placement
    (T = 300)."""
    g = torch.Generator(device="cuda").manual_seed(300 + T)
    x = (torch.randn((T, 2048), generator=g, device="cuda") * 3.0).bfloat16()
    w = (1.0 + 0.1 * torch.randn(2048, generator=g, device="cuda")).bfloat16()
    layer = MoELayer(qwen_layer, top_k=8, norm_weight=w, norm_eps=1e-6)
    logits = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    run = layer.prefill if path == "prefill" else layer.forward
    out, topi, topw = run(x, logits=logits)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    xn = mx.rms_norm_bf16(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6)
    ref = mx.moe_layer(xn, oracle_weights(qwen_layer), topk=8, fast=T > 64)
    assert np.array_equal(logits.cpu().numpy(), ref["logits"])
    assert np.array_equal(topi.cpu().numpy(), ref["idx"])
    o = out.cpu().numpy()
    assert cosine(o, ref["out"]) >= 0.999
    assert max_rel_err(o, ref["out"]) <= 1e-2
    # the same as normalising first and running the unfused layer
    plain = MoELayer(qwen_layer, top_k=8)
    xn_t = torch.from_numpy(xn).bfloat16().cuda()
    out2, topi2, _ = (plain.prefill if path == "prefill" else plain.forward)(xn_t)
    torch.cuda.synchronize()
    assert torch.equal(topi2, topi)
    assert torch.equal(out2, out)
