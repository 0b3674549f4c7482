"""Prefill path of the fused layer (mfi_moe_layer_prefill; mfi_moe_layer for
T * top_k > 4096): compact count-based expert placement and 128-token tcgen05
tiles, vs the kernel-path oracle.

Contract: top-k indices and router logits bit-exact;
layer output max relative error <= 1e-2 and cosine >= 0.999 versus the
fp32-accumulated dequantised reference (the oracle accumulates in float64).
Each (token, slot) output row of the prefill path is rounded to bf16 (as the
reference's prefill rounds y to the activation type,
runtime/model_runner_v2.py:119); the combine then adds them in slot order
with the decode combine's unfused fp32 multiply and add, so a call is
bit-reproducible whatever order the rows were placed in.
"""

import numpy as np
import pytest
import torch

from moe_fused_inference_b200.layer import MoELayer, MoELayerWeights, random_layer_weights
from moe_fused_inference_b200.synthetic import zipf_bias
from oracle import mxfp4 as mx
from tests.conftest import cosine, max_rel_err

pytestmark = pytest.mark.gpu


def oracle_weights(w: MoELayerWeights):
    c = lambda t: t.cpu().numpy()
    return mx.MoELayerWeights(c(w.gate_wp), c(w.gate_sc), c(w.up_wp), c(w.up_sc),
                              c(w.down_wp), c(w.down_sc), c(w.router_wp), c(w.router_sc))


@pytest.fixture(scope="module")
def qwen_layer():
    return random_layer_weights(n_experts=128, hidden=2048, inter=768, std=0.02, seed=5)


def _x(T, seed, H=2048):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((T, H), generator=g, device="cuda").bfloat16()


@pytest.mark.parametrize("T", [1, 37, 300])
def test_prefill_forced_small_T(qwen_layer, T):
    """The prefill kernels on decode sizes (ragged tiles, single tokens)."""
    layer = MoELayer(qwen_layer, top_k=8)
    x = _x(T, 200 + T)
    logits = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    out, topi, topw = layer.prefill(x, logits=logits)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    ref = mx.moe_layer(x.float().cpu().numpy(), oracle_weights(qwen_layer), topk=8, fast=True)
    assert np.array_equal(logits.cpu().numpy(), ref["logits"])
    assert np.array_equal(topi.cpu().numpy(), ref["idx"])
    o = out.cpu().numpy()
    assert cosine(o, ref["out"]) >= 0.999
    assert max_rel_err(o, ref["out"]) <= 1e-2
    # the decode kernels (fp32 rows) on the same input agree to the bf16
    # rounding of the prefill rows: 2^-9 of the largest row, a few 1e-3 of
    # the largest output
    dec, dtopi, _ = layer(x)
    torch.cuda.synchronize()
    assert torch.equal(dtopi, topi)
    assert max_rel_err(o, dec.cpu().numpy()) <= 6e-3


def test_prefill_auto_zipf_T2048(qwen_layer):
    """T = 2048 with the Zipf(1.2) logit skew: mfi_moe_layer
    takes the prefill path on its own; some experts get many 128-token tiles,
    some none."""
    bias = zipf_bias(128, alpha=0.5, seed=3)
    layer = MoELayer(qwen_layer, top_k=8, logit_bias=torch.from_numpy(bias))
    T = 2048
    x = _x(T, 77)
    logits = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    out, topi, topw = layer(x, logits=logits)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    ref = mx.moe_layer(x.float().cpu().numpy(), oracle_weights(qwen_layer), topk=8, fast=True,
                       logit_bias=bias)
    assert np.array_equal(logits.cpu().numpy(), ref["logits"])
    assert np.array_equal(topi.cpu().numpy(), ref["idx"])
    np.testing.assert_allclose(topw.cpu().numpy(), ref["w"], rtol=2e-6, atol=1e-7)
    counts = np.bincount(ref["idx"].ravel(), minlength=128)
    assert counts.max() > 4 * counts.mean()  # the skew is real
    o = out.cpu().numpy()
    assert cosine(o, ref["out"]) >= 0.999
    assert max_rel_err(o, ref["out"]) <= 1e-2


def test_prefill_repeatable_and_capturable(qwen_layer):
    layer = MoELayer(qwen_layer, top_k=8)
    T = 1024
    x = _x(T, 5)
    out = torch.empty((T, 2048), dtype=torch.float32, device="cuda")
    topi = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    topw = torch.empty((T, 8), dtype=torch.float32, device="cuda")
    layer(x, out=out, topi=topi, topw=topw)
    torch.cuda.synchronize()
    first = out.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            layer(x, out=out, topi=topi, topw=topw)
    torch.cuda.current_stream().wait_stream(s)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)  # placement order varies, results do not
    del g


@pytest.mark.parametrize("span", [5, 70])
def test_prefill_router_ragged_tile_and_wide_scales(qwen_layer, span):
    """T = 677 through the tensor-core router (a partial last 128-token tile),
    with every 50th token given 32-element blocks 2^span apart in magnitude.
    span 5: those tokens cannot carry their block scales in the int8 operand,
    so their tiles take the per-block accumulators (fp64 epilogue); span 70:
    beyond the span where that fp64 sum is order-free, so the router
    recomputes them in the fixed order.  Every logit stays bit-exact."""
    T = 677
    x = _x(T, 91).float()
    x[::50, :32] *= 2.0 ** (span // 2 + span % 2)
    x[::50, 32:64] *= 2.0 ** -(span // 2)
    x = x.bfloat16()
    layer = MoELayer(qwen_layer, top_k=8)
    logits = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    out, topi, topw = layer.prefill(x, logits=logits)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    ref = mx.moe_layer(x.float().cpu().numpy(), oracle_weights(qwen_layer), topk=8, fast=True)
    assert np.array_equal(logits.cpu().numpy(), ref["logits"])
    assert np.array_equal(topi.cpu().numpy(), ref["idx"])
    np.testing.assert_allclose(topw.cpu().numpy(), ref["w"], rtol=2e-6, atol=1e-7)
    assert torch.isfinite(out).all()


def test_prefill_zipf_T16384(qwen_layer):
    """BASELINE config 3's headline prefill shape: T = 16384 tokens with the
    Zipf(1.2) logit skew through mfi_moe_layer.  A token's routing and output
    depend only on its own row, so the oracle runs on 2048 of the tokens (every
    8th, spread over every 128-token tile and every expert's tiles): logits
    and top-k bit-exact, weights to rounding, output cosine >= 0.999 and max
    relative error <= 1e-2.  Over all 16384 tokens: no device error, finite
    output, distinct ids per token, weights summing to 1."""
    bias = zipf_bias(128, alpha=0.5, seed=3)
    layer = MoELayer(qwen_layer, top_k=8, logit_bias=torch.from_numpy(bias))
    T = 16384
    x = _x(T, 16384)
    logits = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    out, topi, topw = layer(x, logits=logits)
    torch.cuda.synchronize()
    from moe_fused_inference_b200 import _lib
    assert _lib.load().mfi_device_error(1) == 0
    assert bool(torch.isfinite(out).all())
    ti = topi.cpu().numpy()
    assert (np.sort(ti, axis=1)[:, 1:] != np.sort(ti, axis=1)[:, :-1]).all()
    np.testing.assert_allclose(topw.sum(1).cpu().numpy(), 1.0, rtol=0, atol=1e-5)
    counts = np.bincount(ti.ravel(), minlength=128)
    assert counts.max() > 4 * counts.mean()  # the skew is real: the hottest expert has many tiles
    s = slice(0, T, 8)
    ref = mx.moe_layer(x[s].float().cpu().numpy(), oracle_weights(qwen_layer), topk=8, fast=True,
                       logit_bias=bias)
    assert np.array_equal(logits[s].cpu().numpy(), ref["logits"])
    assert np.array_equal(ti[s], ref["idx"])
    np.testing.assert_allclose(topw[s].cpu().numpy(), ref["w"], rtol=2e-6, atol=1e-7)
    o = out[s].cpu().numpy()
    assert cosine(o, ref["out"]) >= 0.999
    assert max_rel_err(o, ref["out"]) <= 1e-2
