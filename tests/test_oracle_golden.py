"""Pin the CPU oracle to the reference (fixtures generated from the reference's
own Python by tests/golden/make_golden.py) and to its known-answer selftest."""

import hashlib

import numpy as np
import pytest
import torch

from oracle import moe_ref
from oracle import mxfp4 as mx
from tests.conftest import bf16_bits_to_f32


def test_quantizer_cases_bit_exact(golden):
    d = golden("quant_cases.npz")
    for i in range(int(d["n_cases"])):
        p, c = mx.quantize_rows(bf16_bits_to_f32(d[f"x{i}"]))
        assert np.array_equal(p, d[f"p{i}"]), f"packed mismatch in case {i}"
        assert np.array_equal(c, d[f"c{i}"]), f"scale mismatch in case {i}"


def test_quantizer_edge_blocks_bit_exact(golden):
    d = golden("quant_cases.npz")
    p, c = mx.quantize_rows(bf16_bits_to_f32(d["edge_x"]))
    assert np.array_equal(p, d["edge_p"])
    assert np.array_equal(c, d["edge_c"])
    # the 1e-30 floor of the reference's scale rule: tiny blocks get code 28
    assert (d["edge_c"][2] == 28).all() and (d["edge_c"][6] == 28).all()


def _exhaustive_blocks(d):
    amax = bf16_bits_to_f32(d["bits"])
    blk = (amax[:, None] * d["frac"][None, :]).astype(np.float32)
    blk[:, 0] = -amax
    blk[:, 31] = amax
    return mx.bf16_round(blk)


def test_quantizer_exhaustive_bf16_amax(golden):
    """Every positive finite bf16 block maximum: codes and nibbles equal the reference's."""
    d = golden("quant_exhaustive.npz")
    p, c = mx.quantize_rows(_exhaustive_blocks(d))
    assert np.array_equal(c.ravel(), d["codes"])
    assert hashlib.sha256(p.tobytes()).digest() == d["packed_sha256"].tobytes()


def test_scale_rule_matches_reference_numpy_rule_on_all_bf16():
    """The exact frexp rule equals the reference's float32 log2/ceil/overflow rule
    (quant/quantize_mxfp4.py:130-143) for every positive finite bf16 amax."""
    bits = np.arange(1, 0x7F80, dtype=np.uint32)
    amax = (bits << 16).view(np.float32)
    e = np.ceil(np.log2(np.maximum(amax / 6.0, 1e-30))).astype(np.int64)
    s = np.power(2.0, e).astype(np.float32)
    ovf = amax / s > 6.0 + 1e-6
    e[ovf] += 1
    assert np.array_equal(mx.block_exponent(amax), e)


def test_quantizer_f32_inputs(golden):
    d = golden("quant_f32.npz")
    p, c = mx.quantize_rows(d["x"])
    assert np.array_equal(p, d["p"]) and np.array_equal(c, d["c"])


def test_dequant_matches_reference_reconstruct(golden):
    d = golden("dequant.npz")
    assert np.array_equal(mx.dequantize_rows(d["p"], d["c"], 100), d["rec"])


def test_fp4_format_known_answers():
    """Restates the checks of the reference's selftest (quant/fp4_format.py:154-198)."""
    codes = np.arange(16, dtype=np.uint8)
    expected = codes.copy()
    expected[8] = 0  # -0.0 -> +0
    assert np.array_equal(mx.e2m1_code(mx.decode_e2m1(codes)), expected)
    q = lambda v: mx.decode_e2m1(mx.e2m1_code(np.array([v], np.float32)))[0]
    assert q(1.7) == 1.5 and q(0.25) == 0.5 and q(7.0) == 6.0 and q(-3.0) == -3.0
    assert mx.decode_e2m1(np.uint8(0xF)) == -6.0 and mx.decode_e2m1(np.uint8(1)) == 0.5
    for amax, scale in [(5.0, 1.0), (6.0, 1.0), (6.1, 2.0), (12.0, 2.0), (0.5, 0.125)]:
        e = int(mx.block_exponent(np.array([amax], np.float32))[0])
        assert 2.0 ** e == scale
    packed = mx.pack_nibbles(np.array([0x0, 0x7, 0xF, 0x1, 0x3, 0x0], np.uint8))
    assert packed[0] == 0x70 and packed[1] == 0x1F
    assert np.array_equal(mx.unpack_nibbles(packed)[:5], [0x0, 0x7, 0xF, 0x1, 0x3])


def _route_fixture(d):
    E, H, MI, T, K = (int(v) for v in d["dims"])
    st = lambda name: np.stack([d[f"{name}{e}"] for e in range(E)])
    W = mx.MoELayerWeights(st("gate_p"), st("gate_c"), st("up_p"), st("up_c"),
                           st("down_p"), st("down_c"), None, None)
    b2t = lambda u: torch.from_numpy(u.astype(np.int16)).view(torch.bfloat16)
    return W, b2t(d["h"]), b2t(d["wr"]), K


def test_cpu_port_reproduces_reference_moe(golden):
    """oracle.moe_ref (the CPU baseline) = reference ModelRunner.moe_route +
    moe_compute("mxfp4"), bit for bit."""
    d = golden("route_moe.npz")
    W, h, wr, K = _route_fixture(d)
    layer = moe_ref.CpuMoELayer(W, router_bf16=wr, top_k=K)
    out, topi, scores, logits = layer.forward(h)
    assert np.array_equal(logits.float().numpy(), d["logits"])
    assert np.array_equal(topi.numpy(), d["topi"])
    assert np.array_equal(scores.float().numpy(), d["scores"])
    assert np.array_equal(out.float().numpy(), d["out"])


def test_topk_route_matches_reference_topk(golden):
    d = golden("route_moe.npz")
    K = int(d["dims"][4])
    idx, w = mx.topk_route(d["logits"], K)
    assert np.array_equal(idx, d["topi"])
    np.testing.assert_allclose(w, d["scores"], rtol=1e-2)  # reference scores are bf16


def test_topk_tie_breaks_to_lower_index():
    lg = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float32)
    idx, w = mx.topk_route(lg, 3)
    assert idx.tolist() == [[1, 2, 4]]
    np.testing.assert_allclose(w, [[1 / 3, 1 / 3, 1 / 3]], rtol=1e-6)


def test_router_logits_fixed_order_equals_exact_sum():
    """With small dynamic range every partial sum is exact, so the fixed-order
    fp64 logits equal the float64 dot of the dequantised operands."""
    rng = np.random.default_rng(7)
    xq, xs = mx.quantize_rows(mx.bf16_round(rng.standard_normal((3, 2048)).astype(np.float32)))
    wq, ws = mx.quantize_rows(mx.bf16_round(rng.standard_normal((16, 2048)).astype(np.float32) * 0.02))
    lg = mx.router_logits(xq, xs, wq, ws)
    ref = (mx.dequantize_rows(xq, xs).astype(np.float64) @ mx.dequantize_rows(wq, ws).astype(np.float64).T)
    assert np.array_equal(lg, ref.astype(np.float32))


def test_combine_reference_semantics():
    rng = np.random.default_rng(1)
    yd = rng.standard_normal((3 * 4, 5)).astype(np.float32)
    w = rng.random((3, 4)).astype(np.float32)
    out = mx.combine(yd, w, 3)
    ref = np.zeros((3, 5), np.float32)
    for m in range(3):
        for e in range(4):
            ref[m] = (ref[m] + w[m, e] * yd[m * 4 + e]).astype(np.float32)
    assert np.array_equal(out, ref)


def test_kernel_path_layer_close_to_dequantised_reference():
    """The kernel-path oracle vs float64 dequantise-then-matmul of the same
    quantised x and weights with h left unquantised: the only difference is the
    MXFP4 requantisation of h (reference src/ext/mxfp4_decode.cu:252-272),
    which by itself costs about one percent of cosine — the same size as the
    reference's own weight-quantisation error (cos 0.993)."""
    rng = np.random.default_rng(11)
    W = mx.make_layer(rng, n_experts=8, hidden=256, inter=128)
    x = mx.bf16_round(rng.standard_normal((4, 256)).astype(np.float32))
    r = mx.moe_layer(x, W, topk=4)
    xd = mx.dequantize_rows(r["xq"], r["xsc"]).astype(np.float64)
    out = np.zeros((4, 256))
    for t in range(4):
        for s in range(4):
            e = r["idx"][t, s]
            g = xd[t] @ mx.dequantize_rows(W.wg[e], W.sg[e]).T
            u = xd[t] @ mx.dequantize_rows(W.wu[e], W.su[e]).T
            h = g / (1 + np.exp(-g)) * u
            out[t] += r["w"][t, s] * (h @ mx.dequantize_rows(W.wd[e], W.sd[e]).astype(np.float64).T)
    from tests.conftest import cosine
    assert cosine(r["out"], out) > 0.98


def test_torch_cpu_quant_dequant_equals_numpy_oracle():
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(96, 200, generator=g) * 0.02).bfloat16()
    w[0, :32] = 0
    w[1, :32] = 1e-35
    ref = mx.dequantize_rows(*mx.quantize_rows(w.float().numpy()), 200)
    got = moe_ref.quant_dequant_bf16(w)
    assert torch.equal(got, torch.from_numpy(ref).bfloat16())


def test_rms_norm_oracle_matches_reference(golden):
    """The fused RMSNorm's restatement against the reference's own
    model_runner.rms_norm (fixture from tests/golden/make_golden.py, 64 rows
    of 2048 with magnitudes from 2^-8 to 2^8).  The definitions could differ
    only through the rounding of the fp32 sum of squares (torch sums in fp32,
    the library exactly and rounds once); on the fixture every one of the
    131,072 normalised bf16 values is identical."""
    from tests.conftest import bf16_bits_to_f32
    g = golden("rms_norm.npz")
    x, w, y = bf16_bits_to_f32(g["x"]), bf16_bits_to_f32(g["w"]), bf16_bits_to_f32(g["y"])
    got = mx.rms_norm_bf16(x, w, float(g["eps"]))
    assert np.array_equal(got, y)
