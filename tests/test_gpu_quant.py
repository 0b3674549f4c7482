"""GPU activation/weight quantiser vs the oracle and the reference fixtures: bit-exact."""

import hashlib

import numpy as np
import pytest
import torch

from moe_fused_inference_b200 import fp4_ext
from moe_fused_inference_b200.layer import quantize_rows
from oracle import mxfp4 as mx
from tests.conftest import bf16_bits_to_f32

pytestmark = pytest.mark.gpu


def _bf16_cuda(bits):
    return torch.from_numpy(np.asarray(bits).astype(np.int16)).view(torch.bfloat16).cuda()


def test_prequant_reference_cases(golden):
    """Shapes of the reference's prequant test (tests/correctness/test_mxfp4_decode.py:57)
    and its mini checkpoint, bit-exact (the reference only asked > 0.999)."""
    dext = fp4_ext.get_decode_ext()
    d = golden("quant_cases.npz")
    for i in range(int(d["n_cases"])):
        xq, xsc = dext.prequant(_bf16_cuda(d[f"x{i}"]))
        assert np.array_equal(xq.cpu().numpy(), d[f"p{i}"]), i
        assert np.array_equal(xsc.cpu().numpy(), d[f"c{i}"]), i


def test_prequant_edge_blocks(golden):
    d = golden("quant_cases.npz")
    xq, xsc = fp4_ext.get_decode_ext().prequant(_bf16_cuda(d["edge_x"]))
    assert np.array_equal(xq.cpu().numpy(), d["edge_p"])
    assert np.array_equal(xsc.cpu().numpy(), d["edge_c"])


def test_prequant_exhaustive_bf16(golden):
    d = golden("quant_exhaustive.npz")
    amax = bf16_bits_to_f32(d["bits"])
    blk = (amax[:, None] * d["frac"][None, :]).astype(np.float32)
    blk[:, 0] = -amax
    blk[:, 31] = amax
    x = torch.from_numpy(blk).bfloat16().cuda()
    xq, xsc = fp4_ext.get_decode_ext().prequant(x)
    assert np.array_equal(xsc.cpu().numpy().ravel(), d["codes"])
    assert hashlib.sha256(xq.cpu().numpy().tobytes()).digest() == d["packed_sha256"].tobytes()


@pytest.mark.parametrize("shape", [(1, 2048), (64, 2048), (7, 100), (3, 33), (5, 4096), (300, 768)])
def test_quantize_rows_random_bf16(shape):
    g = torch.Generator().manual_seed(shape[0] * 1000 + shape[1])
    x = (torch.randn(shape, generator=g) * 0.5).bfloat16()
    p, c = quantize_rows(x.cuda())
    rp, rc = mx.quantize_rows(x.float().numpy())
    assert np.array_equal(p.cpu().numpy(), rp) and np.array_equal(c.cpu().numpy(), rc)


def test_quantize_rows_f32_and_f16(golden):
    d = golden("quant_f32.npz")
    p, c = quantize_rows(torch.from_numpy(d["x"]).cuda())
    assert np.array_equal(p.cpu().numpy(), d["p"]) and np.array_equal(c.cpu().numpy(), d["c"])
    x16 = torch.from_numpy(d["x"]).half()
    p, c = quantize_rows(x16.cuda())
    rp, rc = mx.quantize_rows(x16.float().numpy())
    assert np.array_equal(p.cpu().numpy(), rp) and np.array_equal(c.cpu().numpy(), rc)


def test_half_roundtrip_matches_binding_cast():
    x = torch.randn(9, 96) * 3
    p, c = quantize_rows(x.cuda(), half_roundtrip=True)
    rp, rc = mx.quantize_rows(mx.f32_to_f16_roundtrip(x.numpy()))
    assert np.array_equal(p.cpu().numpy(), rp) and np.array_equal(c.cpu().numpy(), rc)


def test_weight_quantizer_large_matrix():
    """Expert-sized weights (768 x 2048 bf16 N(0, 0.02)): the device quantiser is
    the reference's quantize_expert_tensor bit for bit."""
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(768, 2048, generator=g) * 0.02).bfloat16()
    p, c = quantize_rows(w.cuda())
    rp, rc = mx.quantize_rows(w.float().numpy())
    assert np.array_equal(p.cpu().numpy(), rp) and np.array_equal(c.cpu().numpy(), rc)


def test_selftest_numerics_all_fp32_patterns():
    """The library's own SwiGLU quotient (Markstein's division) equals CUDA's
    correctly rounded g / (1 + expf(-g)) — the reference build's arithmetic,
    src/ext/mxfp4_decode.cu:258 — and its bit-level E2M1 rounding equals the
    threshold definition, on all 2^32 fp32 bit patterns."""
    from moe_fused_inference_b200 import _lib
    out = torch.zeros(4, dtype=torch.int64, device="cuda")
    lib = _lib.load()
    assert lib.mfi_selftest_numerics(out.data_ptr(), None) == 0, lib.mfi_last_error()
    torch.cuda.synchronize()
    bad_q, bad_m, first_q, first_m = out.tolist()
    assert bad_q == 0, f"{bad_q} quotient mismatches, first at bits {first_q & 0xFFFFFFFF:#010x}"
    assert bad_m == 0, f"{bad_m} E2M1 mismatches, first at bits {first_m & 0xFFFFFFFF:#010x}"
