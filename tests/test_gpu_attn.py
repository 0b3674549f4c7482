"""FP8-KV cache write and decode attention on the GPU against oracle/attn.py.

kv_write is integer work on bytes: bit-exact against the restated reference
encoder on all 65,536 bf16 bit patterns, and against the standard e4m3fn
encoding with per-KV-head scales.  attn_decode is fp32 arithmetic: max
relative error <= 2e-5 against the float64 oracle on the same cache bytes.
Shapes follow the reference's callers: Qwen3-30B-A3B attention (32 query /
4 KV heads, head_dim 128), M = 1 (runtime/model_runner_v3.py:98-129) and the
speculative verify's M = L + 1 = 5 rows (runtime/model_runner_v2.py:244-262).
"""

import numpy as np
import pytest
import torch

from moe_fused_inference_b200 import _lib, fp4_ext
from oracle import attn as oa
from tests.conftest import max_rel_err

pytestmark = pytest.mark.gpu


def _dpos(v):
    return torch.tensor([v], dtype=torch.int32, device="cuda")


def test_kv_write_all_bf16_patterns_reference_codec():
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    k = bits.view(512, 1, 128).cuda()
    v = torch.flip(bits, [0]).contiguous().view(512, 1, 128).cuda()
    kvk = torch.zeros((600, 1, 128), dtype=torch.uint8, device="cuda")
    kvv = torch.zeros_like(kvk)
    dext = fp4_ext.get_decode_ext()
    dext.kv_write(k, v, kvk, kvv, _dpos(40), 512)
    torch.cuda.synchronize()
    kf = k.float().cpu().numpy().reshape(512, 1, 128)
    vf = v.float().cpu().numpy().reshape(512, 1, 128)
    assert np.array_equal(kvk[40:552].cpu().numpy(), oa.e4m3_ref_encode(kf))
    assert np.array_equal(kvv[40:552].cpu().numpy(), oa.e4m3_ref_encode(vf))
    # positions outside [base, base + M) are untouched
    assert int(kvk[:40].abs().sum()) == 0 and int(kvk[552:].abs().sum()) == 0


def test_kv_write_per_head_scales_standard_codec():
    rng = np.random.default_rng(1)
    M, Hkv, D = 7, 4, 128
    x = (rng.standard_normal((2, M, Hkv, D)) * np.array([1, 4, 40, 900])[None, None, :, None])
    k = torch.from_numpy(x[0].astype(np.float32)).bfloat16().cuda()
    v = torch.from_numpy(x[1].astype(np.float32)).bfloat16().cuda()
    ks = torch.tensor([0.01, 0.03, 0.2, 1.0], device="cuda")
    vs = torch.tensor([0.02, 0.05, 0.1, 3.0], device="cuda")
    kvk = torch.zeros((16, Hkv, D), dtype=torch.uint8, device="cuda")
    kvv = torch.zeros_like(kvk)
    fp4_ext.get_decode_ext().kv_write(k, v, kvk, kvv, _dpos(3), M, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    kf, vf = k.float().cpu().numpy(), v.float().cpu().numpy()
    want_k = oa.e4m3_std_encode(kf / ks.cpu().numpy()[None, :, None])
    want_v = oa.e4m3_std_encode(vf / vs.cpu().numpy()[None, :, None])
    assert np.array_equal(kvk[3:3 + M].cpu().numpy(), want_k)
    assert np.array_equal(kvv[3:3 + M].cpu().numpy(), want_v)


def _cache(rng, max_pos, Hkv, D, fill, scales=None):
    k = rng.standard_normal((max_pos, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((max_pos, Hkv, D)).astype(np.float32)
    k[fill:] = 0
    v[fill:] = 0
    if scales is None:
        return oa.e4m3_ref_encode(k), oa.e4m3_ref_encode(v)
    ks, vs = scales
    return (oa.e4m3_std_encode(k / ks[None, :, None]), oa.e4m3_std_encode(v / vs[None, :, None]))


@pytest.mark.parametrize("M,base,max_pos,Hq,Hkv", [
    (1, 0, 64, 32, 4),        # first token: one live position
    (1, 100, 256, 32, 4),
    (5, 1019, 1088, 32, 4),   # speculative verify, L = 4 drafts
    (3, 2046, 2048, 32, 4),   # the last row lies past the cache: zeros
    (1, 4095, 4096, 32, 4),   # long context, many splits
    (2, 77, 300, 16, 1),      # one KV head, 16 query heads
    (4, 31, 33, 8, 8),        # no grouping
])
def test_attn_decode_matches_oracle(M, base, max_pos, Hq, Hkv):
    rng = np.random.default_rng(M * 1000 + base)
    D = 128
    kvk, kvv = _cache(rng, max_pos, Hkv, D, min(base + M, max_pos))
    q = torch.from_numpy(rng.standard_normal((M, Hq, D)).astype(np.float32)).bfloat16().cuda()
    sc = torch.empty((M, Hq, max_pos), dtype=torch.float32, device="cuda")
    o = fp4_ext.get_decode_ext().attn_decode(q, torch.from_numpy(kvk).cuda(),
                                             torch.from_numpy(kvv).cuda(), _dpos(base), sc, M)
    torch.cuda.synchronize()
    assert _lib.load().mfi_device_error(1) == 0
    want = oa.attn_decode(q.float().cpu().numpy(), kvk, kvv, base)
    got = o.cpu().numpy()
    assert max_rel_err(got, want) <= 2e-5
    live = [m for m in range(M) if base + m < max_pos]
    assert np.all(got[len(live):] == 0)


def test_attn_decode_per_head_scales():
    rng = np.random.default_rng(9)
    M, base, max_pos, Hq, Hkv, D = 5, 600, 1024, 32, 4, 128
    ks = np.array([0.004, 0.01, 0.05, 0.2], np.float32)
    vs = np.array([0.003, 0.02, 0.07, 0.5], np.float32)
    kvk, kvv = _cache(rng, max_pos, Hkv, D, base + M, scales=(ks, vs))
    q = torch.from_numpy(rng.standard_normal((M, Hq, D)).astype(np.float32)).bfloat16().cuda()
    o = fp4_ext.get_decode_ext().attn_decode(
        q, torch.from_numpy(kvk).cuda(), torch.from_numpy(kvv).cuda(), _dpos(base), None, M,
        k_scale=torch.from_numpy(ks), v_scale=torch.from_numpy(vs))
    torch.cuda.synchronize()
    want = oa.attn_decode(q.float().cpu().numpy(), kvk, kvv, base, k_scale=ks, v_scale=vs)
    assert max_rel_err(o.cpu().numpy(), want) <= 2e-5


def test_kv_write_attn_graph_replay_with_moving_position():
    """The v3 runner's use (runtime/model_runner_v3.py:98-129): kv_write and
    attn_decode with the stale 5-argument forms (M = 1) captured once in a
    CUDA graph and replayed while the device position advances."""
    rng = np.random.default_rng(3)
    Hq, Hkv, D, max_pos = 32, 4, 128, 64
    dext = fp4_ext.get_decode_ext()
    kvk = torch.zeros((max_pos, Hkv, D), dtype=torch.uint8, device="cuda")
    kvv = torch.zeros_like(kvk)
    dpos = _dpos(0)
    q32 = torch.zeros((Hq, D), dtype=torch.bfloat16, device="cuda")
    k32 = torch.zeros((Hkv, D), dtype=torch.bfloat16, device="cuda")
    v32 = torch.zeros((Hkv, D), dtype=torch.bfloat16, device="cuda")
    sc = torch.zeros((Hq, max_pos), dtype=torch.float32, device="cuda")
    o32 = torch.zeros((1, Hq, D), dtype=torch.float32, device="cuda")

    def body():
        dext.kv_write(k32, v32, kvk, kvv, dpos)
        o32.copy_(dext.attn_decode(q32, kvk, kvv, dpos, sc))

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            body()
    torch.cuda.current_stream().wait_stream(s)
    kvk.zero_()
    kvv.zero_()
    ks, vs = [], []
    for step in range(6):
        dpos.fill_(step)
        qn = rng.standard_normal((Hq, D)).astype(np.float32)
        kn = rng.standard_normal((Hkv, D)).astype(np.float32)
        vn = rng.standard_normal((Hkv, D)).astype(np.float32)
        q32.copy_(torch.from_numpy(qn).bfloat16())
        k32.copy_(torch.from_numpy(kn).bfloat16())
        v32.copy_(torch.from_numpy(vn).bfloat16())
        g.replay()
        torch.cuda.synchronize()
        ks.append(k32.float().cpu().numpy())
        vs.append(v32.float().cpu().numpy())
        kc = np.zeros((max_pos, Hkv, D), np.uint8)
        vc = np.zeros((max_pos, Hkv, D), np.uint8)
        kc[: step + 1] = oa.e4m3_ref_encode(np.stack(ks))
        vc[: step + 1] = oa.e4m3_ref_encode(np.stack(vs))
        assert np.array_equal(kvk.cpu().numpy(), kc)
        want = oa.attn_decode(q32.float().cpu().numpy()[None], kc, vc, step)
        assert max_rel_err(o32.cpu().numpy(), want) <= 2e-5
    del g


@pytest.mark.parametrize("scaled", [False, True])
def test_attn_decode_every_byte_code(scaled):
    """Caches of uniformly random bytes, so every E4M3 code occurs —
    exponent fields 0 and 15 included, where the reference's decoder differs
    from the standard one (m 2^-6, 448 (1 + m/8)).  Small queries keep the
    scores moderate for the 2e-5 bound.  With scales the standard format has
    no value for 0x7F / 0xFF (NaN), so those bytes are left out."""
    rng = np.random.default_rng(77 + scaled)
    M, base, max_pos, Hq, Hkv, D = 2, 300, 400, 32, 4, 128
    kvk = rng.integers(0, 256, (max_pos, Hkv, D)).astype(np.uint8)
    kvv = rng.integers(0, 256, (max_pos, Hkv, D)).astype(np.uint8)
    ks = vs = None
    if scaled:
        for c in (kvk, kvv):
            c[(c & 0x7F) == 0x7F] = 0x11
        ks = np.array([0.5, 0.25, 1.0, 2.0], np.float32)
        vs = np.array([0.125, 1.0, 0.5, 4.0], np.float32)
    q = torch.from_numpy(rng.standard_normal((M, Hq, D)).astype(np.float32) * 0.01).bfloat16().cuda()
    kw = {} if not scaled else {"k_scale": torch.from_numpy(ks), "v_scale": torch.from_numpy(vs)}
    o = fp4_ext.get_decode_ext().attn_decode(q, torch.from_numpy(kvk).cuda(),
                                             torch.from_numpy(kvv).cuda(), _dpos(base), None, M,
                                             **kw)
    torch.cuda.synchronize()
    want = oa.attn_decode(q.float().cpu().numpy(), kvk, kvv, base, k_scale=ks, v_scale=vs)
    assert max_rel_err(o.cpu().numpy(), want) <= 2e-5


def test_attn_decode_batched_sequences():
    """mfi_attn_decode_batched: 6 sequences with their own caches (stride
    between them) and one device position, M = 3 rows each, as the batched
    model runner calls it; every sequence equals its single-sequence oracle."""
    rng = np.random.default_rng(5)
    S, M, base, max_pos, Hq, Hkv, D = 6, 3, 700, 720, 32, 4, 128
    caches = [_cache(rng, max_pos, Hkv, D, base + M) for _ in range(S)]
    kvk = torch.from_numpy(np.stack([c[0] for c in caches])).cuda()
    kvv = torch.from_numpy(np.stack([c[1] for c in caches])).cuda()
    q = torch.from_numpy(rng.standard_normal((S, M, Hq, D)).astype(np.float32)).bfloat16().cuda()
    o = torch.empty((S, M, Hq, D), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    nws = int(lib.mfi_attn_decode_batched_workspace_bytes(S, M, Hq, Hkv, D, max_pos))
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    st = lib.mfi_attn_decode_batched(q.data_ptr(), kvk.data_ptr(), kvv.data_ptr(),
                                     max_pos * Hkv * D, _dpos(base).data_ptr(), o.data_ptr(), S, M,
                                     Hq, Hkv, D, max_pos, None, None, ws.data_ptr(), nws, None)
    assert st == 0, lib.mfi_last_error()
    torch.cuda.synchronize()
    qn = q.float().cpu().numpy()
    for s in range(S):
        want = oa.attn_decode(qn[s], caches[s][0], caches[s][1], base)
        assert max_rel_err(o[s].cpu().numpy(), want) <= 2e-5
