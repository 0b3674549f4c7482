"""The arithmetic of the tensor-core prefill router (route_tc.cu), restated on
the CPU and checked bit for bit against the fixed-order router logits of the
oracle (oracle/mxfp4.py:router_logits, the order of every GPU router).

The kernel relies on two facts, both checked here on seeded inputs:

* fast path: when a row's 64 block codes span at most 3 binades, scaling its
  int8 operand by 2^(code - row minimum) keeps it within [-96, 96]; one
  integer accumulator over all blocks then holds the exact logit in units of
  2^(minx + minw - 256), and a single round-to-nearest int -> fp32 conversion
  gives the fixed-order result;
* per-block path: with exact block products and an exponent span of at most
  28 binades (34 for unscaled operands), fp64 accumulation in any order gives
  the same value as the fixed order.
"""

import numpy as np
import pytest

from oracle import mxfp4 as mx


def _rows(rng, m, k, std, block_scale_span=0):
    x = rng.standard_normal((m, k)).astype(np.float32) * std
    if block_scale_span:
        # each 32-element block scaled by 2^j, j in [0, span]: code spans grow
        s = rng.integers(0, block_scale_span + 1, size=(m, k // 32)).astype(np.float32)
        x = x * np.repeat(np.exp2(s), 32, axis=1)
    return mx.quantize_rows(mx.bf16_round(x))


def _fast_path(xq, xsc, wq, wsc):
    """route_tc_kernel's single-accumulator path: scaled int8 operands, one
    exact integer sum, one rounding."""
    a = mx._int_codes(xq)
    b = mx._int_codes(wq)
    m, kp = a.shape
    n = b.shape[0]
    nb = kp // 32
    sx = xsc.astype(np.int64)
    sw = wsc.astype(np.int64)
    shx = sx - sx.min(axis=1, keepdims=True)
    shw = sw - sw.min(axis=1, keepdims=True)
    assert shx.max() <= 3 and shw.max() <= 3, "rows outside the fast path"
    a8 = a.reshape(m, nb, 32) << shx[:, :, None]
    b8 = b.reshape(n, nb, 32) << shw[:, :, None]
    assert np.abs(a8).max() <= 127 and np.abs(b8).max() <= 127, "operand leaves int8"
    d = np.einsum("mk,nk->mn", a8.reshape(m, kp), b8.reshape(n, kp))
    assert np.abs(d).max() < 2 ** 31, "s32 accumulator overflow"
    k = sx.min(axis=1)[:, None] + sw.min(axis=1)[None, :] - 256
    assert k.min() >= -126 and k.max() <= 96, "result outside the fp32 normal range"
    f = d.astype(np.float32)  # round to nearest
    return np.ldexp(f, k.astype(np.int32)).astype(np.float32)


def _per_block_any_order(xq, xsc, wq, wsc, seed):
    """The per-block path: exact block products added in fp64 in a shuffled
    order."""
    bd = mx.block_dots(xq, xsc, wq, wsc)
    order = np.random.default_rng(seed).permutation(bd.shape[-1])
    acc = np.zeros(bd.shape[:2], dtype=np.float64)
    for b in order:
        acc = acc + bd[:, :, b]
    return acc.astype(np.float32)


@pytest.fixture(scope="module")
def router():
    return _rows(np.random.default_rng(11), 128, 2048, 0.02)


def test_fast_path_equals_fixed_order(router):
    wq, wsc = router
    xq, xsc = _rows(np.random.default_rng(12), 96, 2048, 1.0)
    ref = mx.router_logits(xq, xsc, wq, wsc)
    got = _fast_path(xq, xsc, wq, wsc)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_fast_path_at_the_span_limit(router):
    """Token rows whose block codes span exactly 3 binades still fit."""
    wq, wsc = router
    xq, xsc = _rows(np.random.default_rng(13), 64, 2048, 1.0, block_scale_span=2)
    spans = xsc.max(axis=1).astype(int) - xsc.min(axis=1).astype(int)
    keep = spans <= 3
    assert keep.sum() >= 8 and spans[keep].max() == 3
    xq, xsc = xq[keep], xsc[keep]
    ref = mx.router_logits(xq, xsc, wq, wsc)
    assert np.array_equal(_fast_path(xq, xsc, wq, wsc), ref)


@pytest.mark.parametrize("span", [6, 20])
def test_per_block_fp64_is_order_free(router, span):
    wq, wsc = router
    xq, xsc = _rows(np.random.default_rng(14 + span), 48, 2048, 1.0, block_scale_span=span)
    spans = xsc.max(axis=1).astype(int) - xsc.min(axis=1).astype(int)
    wspan = int((wsc.max(axis=1).astype(int) - wsc.min(axis=1).astype(int)).max())
    assert spans.max() + wspan <= 28
    assert spans.max() > 3  # outside the fast path
    ref = mx.router_logits(xq, xsc, wq, wsc)
    for seed in range(3):
        assert np.array_equal(_per_block_any_order(xq, xsc, wq, wsc, seed), ref)
