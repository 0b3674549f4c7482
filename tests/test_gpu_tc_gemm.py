"""tcgen05 (kind::mxf4) tensor-core GEMM vs the CPU oracle.

The library routes forward()/lin_pq() with M >= 64 rows to the tensor-core
kernel (csrc/tc_gemm.cu).  Reference operator cases:
tests/correctness/test_mxfp4_mma.py:69-100 (expert shapes, K padding) and the
prefill projection shapes of BASELINE config 3 (scaled down in M).
Tolerance: max relative error <= 1e-4 against float64 accumulation of the
dequantised operands (the tensor core accumulates in fp32).
"""

import numpy as np
import pytest
import torch

from moe_fused_inference_b200 import _lib, fp4_ext
from oracle import mxfp4 as mx
from tests.conftest import max_rel_err

pytestmark = pytest.mark.gpu


def make_operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((N, K)).astype(np.float32)
    w *= np.power(2.0, rng.integers(-1, 2, size=(N, 1))).astype(np.float32)
    wp, wc = mx.quantize_rows(mx.bf16_round(w))
    x = rng.standard_normal((M, K)).astype(np.float32) * 0.5
    x[rng.random((M, K)) < 0.005] *= 4.0
    return mx.bf16_round(x), wp, wc


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (64, 8, 64), (200, 300, 100), (256, 512, 2048),
                                   (384, 2048, 768), (130, 96, 256), (1024, 4096, 2048),
                                   (512, 512, 4096),
                                   # N % 4 != 0: the one-tile-per-CTA kernel (tc_gemm_mxf4_kernel)
                                   (200, 301, 256), (64, 150, 2048), (300, 1001, 512)])
def test_tc_forward(M, N, K):
    x, wp, wc = make_operands(M, N, K, seed=M + N + K)
    xh = torch.from_numpy(x).half().cuda()
    y = fp4_ext.get_ext().forward(xh, torch.from_numpy(wp).cuda(), torch.from_numpy(wc).cuda())
    torch.cuda.synchronize()
    assert _lib.load().mfi_device_error(1) == 0, "a bounded wait in the tcgen05 kernel timed out"
    xq, xs = mx.quantize_rows(xh.float().cpu().numpy())
    ref = mx.mx_gemm_deq64(xq, xs, wp, wc)
    assert max_rel_err(y.cpu().numpy(), ref) <= 1e-4


def test_tc_lin_pq_matches_gemv_path():
    """Same operands through the tensor-core path (M = 96) and, row by row, the
    CUDA-core GEMV path (M = 1): both match the oracle."""
    M, N, K = 96, 768, 2048
    x, wp, wc = make_operands(M, N, K, seed=5)
    dext = fp4_ext.get_decode_ext()
    xq, xs = dext.prequant(torch.from_numpy(x).bfloat16().cuda())
    twp, twc = torch.from_numpy(wp).cuda(), torch.from_numpy(wc).cuda()
    y_tc = dext.lin_pq(xq, xs, twp, twc, M, N, K).cpu().numpy()
    y_gv = np.concatenate([dext.lin_pq(xq[i:i + 1], xs[i:i + 1], twp, twc, 1, N, K).cpu().numpy()
                           for i in range(0, M, 17)])
    ref = mx.mx_gemm_deq64(xq.cpu().numpy(), xs.cpu().numpy(), wp, wc)
    assert max_rel_err(y_tc, ref) <= 1e-4
    assert max_rel_err(y_gv, ref[::17]) <= 1e-4


@pytest.mark.parametrize("name,N,K", [("q", 4096, 2048), ("k", 512, 2048), ("o", 2048, 4096)])
def test_dense_projection_T16384(name, N, K):
    """BASELINE config 3's dense projections at their full size, T = 16384
    rows through lin_pq (the persistent tensor-core GEMM; v has k's shape).
    Every row of y depends only on its own activation row, so the float64
    oracle is evaluated on a sample of 264 rows spread over all 128-row tiles
    (every 62nd row, plus the last); the whole output must be finite."""
    M = 16384
    g = torch.Generator(device="cuda").manual_seed(3 + N + K)
    w = (torch.randn((N, K), generator=g, device="cuda") * 0.02).bfloat16()
    x = torch.randn((M, K), generator=g, device="cuda").bfloat16()
    dext = fp4_ext.get_decode_ext()
    wq, wsc = dext.prequant(w)
    xq, xsc = dext.prequant(x)
    y = dext.lin_pq(xq, xsc, wq, wsc, M, N, K)
    torch.cuda.synchronize()
    assert _lib.load().mfi_device_error(1) == 0
    assert bool(torch.isfinite(y).all())
    rows = torch.from_numpy(np.r_[np.arange(0, M, 62), M - 1]).cuda()
    ref = mx.mx_gemm_deq64(xq[rows].cpu().numpy(), xsc[rows].cpu().numpy(), wq.cpu().numpy(),
                           wsc.cpu().numpy())
    assert max_rel_err(y[rows].cpu().numpy(), ref) <= 1e-4
