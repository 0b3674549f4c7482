"""CPU restatement of the FP8-KV decode attention and KV write — TEST
INFRASTRUCTURE ONLY (tests/ may import it; the product path never does).

Restates, in numpy, the reference's graph-friendly attention path
(src/ext/mxfp4_decode.cu:352-490):

* ``e4m3_ref_encode`` — f32_to_e4m3 (mxfp4_decode.cu:447-466): sign from
  x < 0; frexp exponent e of |x|; mantissa q = lround((|x| / 2^(e-1) - 1) * 8)
  (half away from zero), q == 8 carries into the exponent; exponent field
  e + 6; a field <= 0 encodes lround(|x| * 64) clamped to [0, 7]; a field >= 15
  saturates to 0x7F.  (Non-finite inputs are undefined there — lroundf of a
  non-finite value — and map to sign | 0x7F here, as in the library.)
* ``REF_DECODE`` — e4m3_to_f32 (:362-371): exponent 0 -> m * 2^-6, exponent
  15 -> 448 * (1 + m/8), else (1 + m/8) * 2^(e-7).
* ``STD_DECODE`` — the standard e4m3fn values (subnormals m * 2^-9, 0x7F/0xFF
  NaN), used with per-KV-head scales (the library's addition for the
  model configuration's per-head FP8 scale).
* ``attn_decode`` — attn_score_kernel + attn_combine_kernel (:374-421): row m
  of M query rows attends to positions [0, base + m] of its KV head
  (h // (Hq / Hkv)), scores q.k scaled by 1/sqrt(D), softmax, weighted V —
  here in float64, the tolerance reference for the fp32 kernels.

The encoder's semantics are pinned in tests/test_attn_oracle.py against
torch's float8_e4m3fn cast (round to nearest even): the two agree on every
value except exact mantissa ties, where the reference rounds away from zero,
and below 2^-6 and above 2^8, where the reference's format differs.
"""

from __future__ import annotations

import numpy as np


def e4m3_ref_encode(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    sign = np.where(x < 0, 0x80, 0).astype(np.int64)
    with np.errstate(invalid="ignore"):
        a = np.abs(x).astype(np.float64)
    finite = np.isfinite(a)
    a_f = np.where(finite, a, 1.0)
    m, e = np.frexp(a_f)
    eb = e.astype(np.int64) + 6
    man = np.ldexp(a_f, 1 - e)                        # [1, 2), exact
    q = np.floor((man - 1.0) * 8.0 + 0.5).astype(np.int64)  # half away from zero (>= 0)
    carry = q == 8
    q = np.where(carry, 0, q)
    eb = np.where(carry, eb + 1, eb)
    sub = np.clip(np.floor(a_f * 64.0 + 0.5), 0, 7).astype(np.int64)
    sat = eb >= 15
    code = np.where(sat, (15 << 3) | 7, (np.clip(eb, 0, 15) << 3) | q)
    code = np.where(eb <= 0, sub, code)
    code = np.where(a == 0.0, 0, code)
    code = np.where(finite, code, 0x7F)
    return (sign | code).astype(np.uint8)


def _decode_table(ref: bool) -> np.ndarray:
    t = np.empty(256, np.float64)
    for b in range(256):
        m, e = b & 7, (b >> 3) & 15
        if ref:
            if e == 0:
                v = m * 2.0 ** -6
            elif e == 15:
                v = 448.0 * (1.0 + m / 8.0)
            else:
                v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        else:
            if e == 0:
                v = m * 2.0 ** -9
            elif e == 15 and m == 7:
                v = np.nan
            else:
                v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        t[b] = -v if b & 0x80 else v
    return t


REF_DECODE = _decode_table(True)
STD_DECODE = _decode_table(False)


def e4m3_std_encode(x) -> np.ndarray:
    """Standard e4m3fn, round to nearest even, saturating at +-448 (NaN ->
    0x7F): torch's float8_e4m3fn cast of the clamped value."""
    import torch
    t = torch.from_numpy(np.asarray(x, np.float32).copy())
    nan = torch.isnan(t)
    t = torch.clamp(t, -448.0, 448.0)
    out = t.to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    out[nan.numpy()] = 0x7F
    return out


def attn_decode(q, kvk, kvv, base: int, k_scale=None, v_scale=None) -> np.ndarray:
    """q (M, Hq, D) float32 (bf16 values); kvk/kvv uint8 (max_pos, Hkv, D).
    Returns o (M, Hq, D) float64; rows with no live position are zero."""
    q = np.asarray(q, np.float64)
    M, Hq, D = q.shape
    max_pos, Hkv, _ = kvk.shape
    G = Hq // Hkv
    if k_scale is None:
        K = REF_DECODE[kvk]
        V = REF_DECODE[kvv]
    else:
        K = STD_DECODE[kvk] * np.asarray(k_scale, np.float64)[None, :, None]
        V = STD_DECODE[kvv] * np.asarray(v_scale, np.float64)[None, :, None]
    o = np.zeros((M, Hq, D), np.float64)
    for m in range(M):
        pos = base + m
        if base < 0 or pos >= max_pos:
            continue
        S = pos + 1
        for h in range(Hq):
            g = h // G
            s = K[:S, g] @ q[m, h] / np.sqrt(D)
            p = np.exp(s - s.max())
            o[m, h] = (p / p.sum()) @ V[:S, g]
    return o
