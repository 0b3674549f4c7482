"""CPU checks of the FP8 KV-cache oracle (oracle/attn.py).

The reference's E4M3 codec lives only in its sm_120a CUDA source
(src/ext/mxfp4_decode.cu:362-371 decoder, :447-466 encoder), so it cannot be
run here.  The restatement is pinned two ways: known answers derived by hand
from those lines, and agreement with torch's float8_e4m3fn cast (what the
reference's torch attention path, runtime/model_runner_v2.py:175-177, writes)
on every bf16 value in the range where the two formats coincide, except
exact mantissa ties, which the reference rounds away from zero.
"""

import numpy as np
import torch

from oracle import attn as oa


def test_reference_encoder_known_answers():
    cases = {
        1.0: 0x38, -1.0: 0xB8, 1.5: 0x3C, 240.0: 0x77,
        250.0: 0x7F,        # rounds to 2^8: saturates
        448.0: 0x7F, -1000.0: 0xFF,
        2.0 ** -6: 0x08,    # smallest normal of the format
        0.01: 0x01,         # below 2^-6: round(0.64) = 1
        0.005: 0x00,        # round(0.32) = 0
        0.0: 0x00, -0.0: 0x00,  # -0.0 < 0 is false: no sign bit
        1.0625: 0x39,       # mantissa tie (0.5): away from zero (RNE would keep 0x38)
        1.1875: 0x3A,       # tie 1.5 -> 2
        0.0155: 0x08,       # just below 2^-6: the mantissa carry lifts it to 2^-6
        float("inf"): 0x7F, float("-inf"): 0xFF, float("nan"): 0x7F,
    }
    x = np.array(list(cases), np.float32)
    got = oa.e4m3_ref_encode(x)
    want = np.array(list(cases.values()), np.uint8)
    assert np.array_equal(got, want), [(float(a), hex(b), hex(c)) for a, b, c in zip(x, got, want) if b != c]


def test_reference_encoder_matches_rne_except_ties():
    bits = np.arange(65536, dtype=np.uint32)
    x = (bits << 16).view(np.float32)
    a = np.abs(x)
    rng = np.isfinite(x) & (a >= 2.0 ** -6) & (a <= 240.0)
    xs = x[rng]
    ref = oa.e4m3_ref_encode(xs)
    rne = torch.from_numpy(xs.copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    # exact ties: the bf16 mantissa bits below the 3 kept ones are 1000
    m7 = (xs.view(np.uint32) >> 16) & 0x7F
    tie = (m7 & 0xF) == 0x8
    assert np.array_equal(ref[~tie], rne[~tie])
    # at a tie the reference rounds away from zero: one code above RNE when
    # RNE kept the even mantissa
    up = ref[tie].astype(int) - rne[tie].astype(int)
    assert set(np.unique(up)) <= {0, 1}
    assert (up == 1).sum() > 0


def test_decode_tables():
    # normal exponents 1..14: both formats decode alike
    for b in range(256):
        e = (b >> 3) & 15
        if 1 <= e <= 14:
            assert oa.REF_DECODE[b] == oa.STD_DECODE[b]
    # the reference's exponent-0 values are 8x the standard subnormals
    for m in range(8):
        assert oa.REF_DECODE[m] == 8 * oa.STD_DECODE[m]
    # standard table equals torch's float8_e4m3fn decoding
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).double().numpy()
    both = ~np.isnan(t)
    assert np.array_equal(t[both], oa.STD_DECODE[both])
    # encode -> decode round trip of the reference codec on its own grid
    codes = np.array([b for b in range(256) if ((b >> 3) & 15) not in (0, 15)], np.uint8)
    assert np.array_equal(oa.e4m3_ref_encode(oa.REF_DECODE[codes].astype(np.float32)), codes)


def test_attention_oracle_softmax_properties():
    rng = np.random.default_rng(0)
    M, Hq, Hkv, D, max_pos = 3, 8, 2, 128, 40
    q = rng.standard_normal((M, Hq, D)).astype(np.float32)
    v = rng.standard_normal((max_pos, Hkv, D)).astype(np.float32)
    kvk = oa.e4m3_ref_encode(np.zeros_like(v))  # all-zero keys: uniform attention
    kvv = oa.e4m3_ref_encode(v)
    base = 10
    o = oa.attn_decode(q, kvk, kvv, base)
    V = oa.REF_DECODE[kvv]
    for m in range(M):
        want = V[: base + m + 1].mean(axis=0)  # (Hkv, D)
        for h in range(Hq):
            np.testing.assert_allclose(o[m, h], want[h // (Hq // Hkv)], rtol=1e-12, atol=1e-12)
    # rows past the cache get zeros
    o2 = oa.attn_decode(q, kvk, kvv, max_pos - 1)
    assert np.all(o2[1:] == 0) and np.any(o2[0] != 0)
