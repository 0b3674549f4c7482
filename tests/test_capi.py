"""The C ABI library loads and exports every function include/moe_fp4.h declares,
and the Python binding's argument checks behave like the reference binding's
TORCH_CHECKs (no GPU needed: nothing here launches a kernel)."""

import os
import re
import ctypes

import pytest
import torch

from moe_fused_inference_b200 import _lib, build, fp4_ext

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "moe_fp4.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mfi_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    return _lib.load()


def test_header_declares_expected_surface():
    names = declared_functions()
    for must in ["mfi_prequant", "mfi_lin_pq", "mfi_mxfp4_linear", "mfi_moe_gateup",
                 "mfi_moe_down", "mfi_moe_combine", "mfi_moe_layer", "mfi_quantize_rows"]:
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_functions():
        assert hasattr(raw, name), f"{name} missing from libmoe_fp4.so"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_workspace_queries_are_pure_host(lib):
    assert lib.mfi_version() == 3
    assert lib.mfi_moe_layer_workspace_bytes(64, 2048, 768, 128, 8) > 64 * 8 * 2048 * 4
    assert lib.mfi_moe_gateup_workspace_bytes(8, 1) >= 16 * (24 + 16)
    assert lib.mfi_linear_workspace_bytes(16, 256, 2048) >= 16 * (1024 + 64)


def test_argument_errors_report_status_and_message(lib):
    st = lib.mfi_quantize_rows(None, 9, 0, 0, None, None, 1, 32, 32, None)
    assert st == 1
    assert b"dtype" in lib.mfi_last_error()
    st = lib.mfi_lin_pq(None, None, None, None, None, 1, 8, 64, 48, None, 0, None)
    assert st == 1 and b"Kp" in lib.mfi_last_error()
    with pytest.raises(_lib.MfiError):
        _lib.check(lib.mfi_moe_combine(None, 4, None, 0, None, 1, 4, None), "moe_combine")


def test_binding_checks_mirror_reference_messages(lib):
    dext = fp4_ext.get_decode_ext()
    ext = fp4_ext.get_ext()
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="x must be cuda"):
        dext.prequant(x)
    with pytest.raises(RuntimeError, match="x must be cuda"):
        ext.forward(x, torch.zeros(8, 32, dtype=torch.uint8), torch.zeros(8, 2, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="wps must be 2E\\*M"):
        dext.moe_gateup(x, x, [x], [x], 8, 1, 768, 2048)
    with pytest.raises(RuntimeError, match="wps must be E\\*M"):
        dext.moe_down(torch.zeros(8, 10), [x], [x], 8, 1, 2048, 5)
    with pytest.raises(RuntimeError, match="w \\(M,E\\)"):
        dext.moe_combine(torch.zeros(8, 4), torch.zeros(7), 2)
    with pytest.raises(RuntimeError, match="yd \\(M\\*E,N\\)"):
        dext.moe_combine(torch.zeros(6, 4), torch.zeros(8), 1)
    d = torch.zeros(1, dtype=torch.int32)
    kv = torch.zeros(16, 4, 128, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="tensors must be cuda"):
        dext.attn_decode(torch.zeros(1, 32, 128, dtype=torch.bfloat16), kv, kv, d, None, 1)
    with pytest.raises(RuntimeError, match="k and v must be bfloat16"):
        dext.kv_write(torch.zeros(1, 4, 128), torch.zeros(1, 4, 128), kv, kv, d, 1)


def test_weights_struct_layout_matches_header(tmp_path):
    """The ctypes mirror of mfi_moe_weights (the layer's C-ABI argument) has
    the header's field offsets and size: a C probe compiled with gcc prints
    them."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    fields = [f for f, _ in _lib.MoEWeights._fields_]
    src = tmp_path / "probe.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "moe_fp4.h"\nint main(void) {\n'
        + "".join(f'  printf("{f} %zu\\n", offsetof(mfi_moe_weights, {f}));\n' for f in fields)
        + '  printf("sizeof %zu\\n", sizeof(mfi_moe_weights));\n  return 0;\n}\n')
    exe = tmp_path / "probe"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run([gcc, "-I", inc, str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    for f in fields:
        assert int(out[f]) == getattr(_lib.MoEWeights, f).offset, f
    assert int(out["sizeof"]) == ctypes.sizeof(_lib.MoEWeights)
