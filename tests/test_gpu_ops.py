"""Drop-in operators (fp4_ext) on the GPU vs the CPU oracle.

Cases follow the reference's operator tests: tests/correctness/test_mxfp4_mma.py:69-100
(M,N,K incl. K = 100 / 40 padding, M = 1, multi-tile, expert shapes) and
tests/correctness/test_mxfp4_decode.py:76-147 (lin_pq shapes, grouped MoE with
E = 8, N = 768, K = 2048).  Tolerances: GEMM outputs vs the float64-accumulated
dequantised oracle, max relative error <= 1e-4 (the kernel sums exact block
products in fp32); layer-level chains <= 1e-2 and cosine >= 0.999.
"""

import numpy as np
import pytest
import torch

from moe_fused_inference_b200 import fp4_ext
from oracle import mxfp4 as mx
from tests.conftest import cosine, max_rel_err

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-4


def make_w(rng, n, k):
    w = rng.standard_normal((n, k)).astype(np.float32)
    w *= np.power(2.0, rng.integers(-1, 2, size=(n, 1))).astype(np.float32)
    p, c = mx.quantize_rows(mx.bf16_round(w))
    return p, c, torch.from_numpy(p).cuda(), torch.from_numpy(c).cuda()


def make_x(rng, m, k, outliers=0.005):
    x = rng.standard_normal((m, k)).astype(np.float32) * 0.5
    x[rng.random((m, k)) < outliers] *= 4.0
    return mx.bf16_round(x)


@pytest.mark.parametrize("M,N,K", [(16, 8, 64), (16, 8, 100), (16, 8, 40), (1, 8, 64), (1, 32, 64),
                                   (32, 32, 64), (8, 64, 2048), (1, 768, 2048), (8, 2048, 768),
                                   (130, 96, 256)])
def test_forward_mxfp4_linear(M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    wp, wc, twp, twc = make_w(rng, N, K)
    x = make_x(rng, M, K)
    xh = torch.from_numpy(x).half().cuda()
    y = fp4_ext.get_ext().forward(xh, twp, twc).cpu().numpy()
    xq, xsc = mx.quantize_rows(xh.float().cpu().numpy())
    ref = mx.mx_gemm_f64(xq, xsc, wp, wc)
    assert y.shape == (M, N) and y.dtype == np.float32
    assert max_rel_err(y, ref) <= GEMM_TOL
    # bf16 input is rounded through fp16 like the reference binding
    yb = fp4_ext.get_ext().forward(torch.from_numpy(x).bfloat16().cuda(), twp, twc).cpu().numpy()
    assert max_rel_err(yb, ref) <= GEMM_TOL


@pytest.mark.parametrize("M,N,K", [(1, 32, 64), (1, 768, 2048), (1, 2048, 768), (3, 128, 100),
                                   (1, 4096, 2048), (2, 2048, 2048), (64, 128, 2048),
                                   # the streaming GEMV (M <= 8, K % 512 == 0): partial last
                                   # tile, two-stage ring at K = 4096, several tiles per CTA
                                   (7, 999, 2048), (8, 1000, 4096), (3, 20000, 2048),
                                   # the persistent prefill GEMM (N % 4 == 0): one partial
                                   # K tile; several tiles per CTA with every accumulator
                                   # reused; a partial last weight tile
                                   (300, 384, 100), (4700, 2048, 256), (200, 1000, 512),
                                   # the one-tile-per-CTA tensor-core GEMM (M >= 64 and
                                   # N % 4 != 0): partial weight tiles, rows not a multiple of 4
                                   (200, 301, 256), (64, 150, 2048)])
def test_lin_pq(M, N, K):
    rng = np.random.default_rng(1 + M + N + K)
    wp, wc, twp, twc = make_w(rng, N, K)
    x = make_x(rng, M, K)
    dext = fp4_ext.get_decode_ext()
    xq, xsc = dext.prequant(torch.from_numpy(x).bfloat16().cuda())
    y = dext.lin_pq(xq, xsc, twp, twc, M, N, K).cpu().numpy()
    ref = mx.mx_gemm_f64(xq.cpu().numpy(), xsc.cpu().numpy(), wp, wc)
    assert max_rel_err(y, ref) <= GEMM_TOL


def _experts(rng, E, N, K):
    g = [make_w(rng, N, K) for _ in range(E)]
    u = [make_w(rng, N, K) for _ in range(E)]
    d = [make_w(rng, K, N) for _ in range(E)]
    return g, u, d


@pytest.mark.parametrize("M", [1, 4, 5])
def test_moe_gateup_down_combine_chain(M):
    """Grouped chain with the reference's pointer-table order
    (runtime/model_runner_v2.py:279-289), M tokens, E = 8 slots, shared experts.
    Tables of at most 64 entries (M <= 4 for gate/up, M <= 8 for down) are
    grouped inside the tensor-core kernel; larger ones by build_groups_kernel."""
    rng = np.random.default_rng(2 + M)
    E, N, K, NE = 8, 768, 2048, 12
    g, u, d = _experts(rng, NE, N, K)
    ids = np.stack([rng.choice(NE, E, replace=False) for _ in range(M)])
    x = make_x(rng, M, K)
    dext = fp4_ext.get_decode_ext()
    xq, xsc = dext.prequant(torch.from_numpy(x).bfloat16().cuda())
    gwp, gsc, dwp, dsc = [], [], [], []
    for m in range(M):
        gwp += [g[e][2] for e in ids[m]] + [u[e][2] for e in ids[m]]
        gsc += [g[e][3] for e in ids[m]] + [u[e][3] for e in ids[m]]
        dwp += [d[e][2] for e in ids[m]]
        dsc += [d[e][3] for e in ids[m]]
    gu = dext.moe_gateup(xq, xsc, gwp, gsc, E, M, N, K)
    yd = dext.moe_down(gu, dwp, dsc, E, M, K, N)
    w = torch.softmax(torch.from_numpy(rng.standard_normal((M, E)).astype(np.float32)), -1).cuda()
    out = dext.moe_combine(yd, w, M)
    assert gu.shape == (M * E, 2 * N) and yd.shape == (M * E, K) and out.shape == (M, K)

    xqn, xsn = xq.cpu().numpy(), xsc.cpu().numpy()
    gu_n, yd_n = gu.cpu().numpy(), yd.cpu().numpy()
    for m in range(M):
        for s in range(E):
            e = ids[m, s]
            row = m * E + s
            rg = mx.mx_gemm_f64(xqn[m:m + 1], xsn[m:m + 1], g[e][0], g[e][1])[0]
            ru = mx.mx_gemm_f64(xqn[m:m + 1], xsn[m:m + 1], u[e][0], u[e][1])[0]
            assert max_rel_err(gu_n[row, :N], rg) <= GEMM_TOL
            assert max_rel_err(gu_n[row, N:], ru) <= GEMM_TOL
            # down from the GPU's own g/u: identical h, identical requantisation
            h = mx.silu_mul(gu_n[row:row + 1, :N], gu_n[row:row + 1, N:])
            hq, hs = mx.quantize_rows(h)
            rd = mx.mx_gemm_f64(hq, hs, d[e][0], d[e][1])[0]
            assert max_rel_err(yd_n[row], rd) <= GEMM_TOL
    ref_out = mx.combine(yd_n, w.cpu().numpy(), M)
    assert np.array_equal(out.cpu().numpy(), ref_out), "combine must be bit-exact"


def test_moe_tab_variants_and_legacy_arity():
    rng = np.random.default_rng(9)
    E, N, K = 8, 256, 512
    g, u, d = _experts(rng, E, N, K)
    x = make_x(rng, 1, K)
    dext = fp4_ext.get_decode_ext()
    xq, xsc = dext.prequant(torch.from_numpy(x).bfloat16().cuda())
    gw = [t[2] for t in g] + [t[2] for t in u]
    gs = [t[3] for t in g] + [t[3] for t in u]
    gu = dext.moe_gateup(xq, xsc, gw, gs, E, 1, N, K)
    tab = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")
    gu2 = dext.moe_gateup_tab(xq, xsc, tab(gw), tab(gs), E, 1, N, K)
    assert torch.equal(gu, gu2)
    dw = [t[2] for t in d]
    ds = [t[3] for t in d]
    yd = dext.moe_down(gu, dw, ds, E, 1, K, N)
    yd_legacy = dext.moe_down(gu, dw, ds, E, K, N)          # stale 6-argument form
    yd_tab = dext.moe_down_tab(gu, tab(dw), tab(ds), E, 1, K, N)
    assert torch.equal(yd, yd_legacy) and torch.equal(yd, yd_tab)
    w = torch.softmax(torch.randn(E), 0).cuda()
    assert torch.equal(dext.moe_combine(yd, w), dext.moe_combine(yd, w.view(1, E), 1))


@pytest.mark.parametrize("N,K,M", [(64, 128, 20), (128, 256, 4), (128, 256, 20)])
def test_all_tokens_one_expert_and_duplicates(N, K, M):
    """Edge case: every token picks the same experts (one weight shared by all
    entries) — each weight is streamed once for all its tokens.  K = 128 runs
    the CUDA-core GEMV; K = 256 the tensor-core kernel, with the tables grouped
    inside it (M = 4: 32 entries) or by build_groups_kernel (M = 20)."""
    rng = np.random.default_rng(5)
    E = 4
    g, u, d = _experts(rng, E, N, K)
    x = make_x(rng, M, K)
    dext = fp4_ext.get_decode_ext()
    xq, xsc = dext.prequant(torch.from_numpy(x).bfloat16().cuda())
    gw, gs = [], []
    for m in range(M):
        gw += [g[e][2] for e in range(E)] + [u[e][2] for e in range(E)]
        gs += [g[e][3] for e in range(E)] + [u[e][3] for e in range(E)]
    gu = dext.moe_gateup(xq, xsc, gw, gs, E, M, N, K).cpu().numpy()
    for m in range(M):
        for e in range(E):
            ref = mx.mx_gemm_f64(xq.cpu().numpy()[m:m + 1], xsc.cpu().numpy()[m:m + 1], g[e][0], g[e][1])[0]
            assert max_rel_err(gu[m * E + e, :N], ref) <= GEMM_TOL


def test_combine_caps_at_eight_slots_like_reference():
    yd = torch.randn(2 * 10, 33).cuda()
    w = torch.rand(2, 10).cuda()
    out = fp4_ext.get_decode_ext().moe_combine(yd, w, 2).cpu().numpy()
    ref = mx.combine(yd.cpu().numpy().reshape(2, 10, 33)[:, :8].reshape(16, 33),
                     w.cpu().numpy()[:, :8], 2)
    assert np.array_equal(out, ref)
