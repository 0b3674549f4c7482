"""mfi_mxfp4_linear_noalloc — the allocation-free form of mxfp4_linear.

It exists for callers that cannot allocate device memory (a plugin whose host
program owns all GPU memory, an FFI caller without the framework's allocator,
a hot path that must not call cudaMalloc): its scratch is a 4 MiB static
device array inside the library instead of a caller workspace.  This test
calls it through the C ABI twice in a row — a tensor-core-sized call, then a
GEMV-sized call with another K that finds the first call's leftovers in the
shared array — and compares each result with the workspace entry point
mfi_mxfp4_linear on the same inputs (max relative error <= 1e-4, the GEMM
tolerance of the other tests).  It runs last in the suite (file name) and
also passes alone in a fresh process, where its first call sets up the array.
"""

import numpy as np
import pytest
import torch

from moe_fused_inference_b200 import _lib
from moe_fused_inference_b200.layer import quantize_rows
from tests.conftest import max_rel_err

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (torch.randn((N, K), generator=g, device="cuda") * 0.02).bfloat16()
    wp, wsc = quantize_rows(w)
    x = torch.randn((M, K), generator=g, device="cuda").bfloat16()
    return x, wp, wsc


def _with_workspace(lib, x, wp, wsc, M, N, K, Kp, stream):
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.mfi_linear_workspace_bytes(M, N, Kp), dtype=torch.uint8, device="cuda")
    _lib.check(lib.mfi_mxfp4_linear(x.data_ptr(), _lib.MFI_BF16, K, wp.data_ptr(), wsc.data_ptr(),
                                    y.data_ptr(), M, N, Kp, ws.data_ptr(), ws.numel(), stream),
               "mxfp4_linear")
    return y


def _no_alloc(lib, x, wp, wsc, M, N, K, Kp, stream):
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    _lib.check(lib.mfi_mxfp4_linear_noalloc(x.data_ptr(), _lib.MFI_BF16, K, wp.data_ptr(),
                                            wsc.data_ptr(), y.data_ptr(), M, N, Kp, stream),
               "mxfp4_linear_noalloc")
    return y


def test_noalloc_linear_two_calls_match_workspace_entry_point():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for M, N, K, seed in [(160, 512, 2048, 1), (5, 768, 768, 2)]:
        Kp = (K + 31) // 32 * 32
        x, wp, wsc = _operands(M, N, K, seed)
        y_ref = _with_workspace(lib, x, wp, wsc, M, N, K, Kp, stream)
        y = _no_alloc(lib, x, wp, wsc, M, N, K, Kp, stream)
        torch.cuda.synchronize()
        assert max_rel_err(y.cpu().numpy(), y_ref.cpu().numpy()) <= 1e-4, (M, N, K)
    assert lib.mfi_device_error(1) == 0


def test_noalloc_linear_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    M, N, K = 8192, 4096, 4096  # needs far more than the 4 MiB static array
    y = torch.empty((1, 1), dtype=torch.float32, device="cuda")
    st = lib.mfi_mxfp4_linear_noalloc(y.data_ptr(), _lib.MFI_BF16, K, y.data_ptr(), y.data_ptr(),
                                      y.data_ptr(), M, N, K, torch.cuda.current_stream().cuda_stream)
    assert st == 3
    assert b"4 MiB" in lib.mfi_last_error()
