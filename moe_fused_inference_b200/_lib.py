"""ctypes binding of libmoe_fp4.so (C ABI declared in include/moe_fp4.h).

The library is built in-tree by ``python -m moe_fused_inference_b200.build``
(``__graft_entry__.build()`` does it too).  There is no fallback: if the
shared object is missing or fails to load, every operator raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libmoe_fp4.so")

_lock = threading.Lock()
_lib = None

# Every symbol include/moe_fp4.h declares: name -> (restype, argtypes).
_VP = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t
SIGNATURES = {
    "mfi_last_error": (ctypes.c_char_p, []),
    "mfi_version": (_I, []),
    "mfi_prequant": (_I, [_VP, _VP, _VP, _I, _I, _I, _VP]),
    "mfi_quantize_rows": (_I, [_VP, _I, _LL, _I, _VP, _VP, _I, _I, _I, _VP]),
    "mfi_device_error": (_I, [_I]),
    "mfi_selftest_numerics": (_I, [_VP, _VP]),
    "mfi_lin_pq_workspace_bytes": (_SZ, [_I, _I, _I]),
    "mfi_lin_pq": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP, _SZ, _VP]),
    "mfi_linear_workspace_bytes": (_SZ, [_I, _I, _I]),
    "mfi_mxfp4_linear": (_I, [_VP, _I, _I, _VP, _VP, _VP, _I, _I, _I, _VP, _SZ, _VP]),
    "mfi_mxfp4_linear_noalloc": (_I, [_VP, _I, _I, _VP, _VP, _VP, _I, _I, _I, _VP]),
    "mfi_moe_gateup_workspace_bytes": (_SZ, [_I, _I]),
    "mfi_moe_gateup": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP, _SZ, _VP]),
    "mfi_moe_down_workspace_bytes": (_SZ, [_I, _I, _I]),
    "mfi_moe_down": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP, _SZ, _VP]),
    "mfi_moe_combine": (_I, [_VP, _I, _VP, _I, _VP, _I, _I, _VP]),
    "mfi_kv_write": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP, _VP, _VP]),
    "mfi_attn_decode_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "mfi_attn_decode": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP, _VP, _VP, _SZ,
                             _VP]),
    "mfi_attn_decode_batched_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "mfi_attn_decode_batched": (_I, [_VP, _VP, _VP, _LL, _VP, _VP, _I, _I, _I, _I, _I, _I, _VP,
                                     _VP, _VP, _SZ, _VP]),
    "mfi_moe_prepared_bytes": (_SZ, [_I, _I, _I]),
    "mfi_moe_prepare": (_I, [_VP, _VP, _SZ, _VP]),
    "mfi_moe_layer_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "mfi_moe_layer_init_workspace": (_I, [_VP, _SZ, _I, _I, _I, _I, _I, _VP]),
    "mfi_moe_layer": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "mfi_moe_layer_ex": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _SZ, _VP, _I, _VP]),
    "mfi_moe_route": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _VP]),
    "mfi_moe_route_workspace_bytes": (_SZ, [_I, _I, _I]),
    "mfi_moe_route_ex": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "mfi_moe_layer_prefill_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "mfi_moe_layer_prefill": (_I, [_VP, _VP, _I, _VP, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "mfi_moe_experts_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "mfi_moe_experts": (_I, [_VP, _VP, _LL, _VP, _LL, _VP, _LL, _VP, _LL, _I, _VP, _LL, _VP, _SZ,
                             _VP]),
    "mfi_ep_row_bytes": (_I, [_I, _I]),
    "mfi_ep_pack": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _VP, _VP, _VP, _VP]),
    "mfi_ep_mask_recv": (_I, [_VP, _I, _I, _I, _I, _VP]),
    "mfi_ep_unpack": (_I, [_VP, _VP, _I, _I, _I, _I, _VP, _VP]),
    "mfi_ipc_alloc": (_I, [_SZ, ctypes.POINTER(_VP)]),
    "mfi_ipc_free": (_I, [_VP]),
    "mfi_ipc_handle": (_I, [_VP, _VP]),
    "mfi_ipc_open": (_I, [_VP, ctypes.POINTER(_VP)]),
    "mfi_ipc_close": (_I, [_VP]),
    "mfi_copy_async": (_I, [_VP, _VP, _SZ, _VP]),
    "mfi_ep_flag_bytes": (_SZ, []),
    "mfi_ep_recv_bytes": (_SZ, [_I, _I, _I, _I]),
    "mfi_ep_ret_bytes": (_SZ, [_I, _I, _I]),
    "mfi_ep_table_bytes": (_SZ, []),
    "mfi_ep_table_set": (_I, [_VP, _I, _VP, _VP, _VP]),
    "mfi_ep_route_dispatch": (_I, [_VP, _VP, _I, _I, _I, _I, _VP, _VP, _VP, _VP, _VP, _VP]),
    "mfi_ep_experts_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "mfi_ep_experts_return": (_I, [_VP, _I, _I, _I, _VP, _VP, _VP, _VP, _SZ, _VP]),
    "mfi_ep_unpack_wait": (_I, [_I, _I, _I, _I, _VP, _VP, _VP, _VP, _VP]),
}

MFI_F32, MFI_F16, MFI_BF16 = 0, 1, 2


class MoEWeights(ctypes.Structure):
    """Mirror of ``mfi_moe_weights`` (include/moe_fp4.h)."""

    _fields_ = [
        ("gate_wp", _VP), ("gate_sc", _VP), ("up_wp", _VP), ("up_sc", _VP),
        ("down_wp", _VP), ("down_sc", _VP), ("router_wp", _VP), ("router_sc", _VP),
        ("n_experts", _I), ("hidden", _I), ("inter", _I), ("top_k", _I),
        ("prepared", _VP), ("logit_bias", _VP), ("norm_weight", _VP),
        ("norm_eps", ctypes.c_float),
    ]


class MfiError(RuntimeError):
    """A libmoe_fp4 call returned a non-zero status."""


class MfiDeviceError(MfiError):
    """A kernel of the library reported a failure through the device error flag."""


# Codes of the device error flag (mfi_device_error): the first failure of any
# kernel on the device since the flag was last cleared.
DEVICE_ERRORS = {
    1: "a load producer's bounded wait timed out",
    2: "an MMA issuer's bounded wait timed out",
    3: "an epilogue's bounded wait timed out",
    4: "a down item's wait for its h rows timed out, or an expert id was out of range",
    5: "an expert region overflowed: duplicate expert ids or a workspace whose counters "
       "were not initialised",
    6: "the router rows did not arrive in time",
    7: "a peer rank's dispatch did not arrive in time",
    8: "a peer rank's return did not arrive in time",
    9: "a received exchange block's row count was outside [0, capacity] (treated as empty)",
}

# MFI_CHECK_DEVICE=1: every checked call synchronises the device and raises
# MfiDeviceError if the flag is set (a debugging aid: it serialises the host
# with the GPU after every operator).
_CHECK_DEVICE = os.environ.get("MFI_CHECK_DEVICE", "0") == "1"


def device_error(clear: bool = True) -> int:
    """Read (and by default clear) the device error flag of the current
    device; synchronous.  0 means no kernel has reported a failure."""
    v = int(load().mfi_device_error(1 if clear else 0))
    if v < 0:
        raise MfiError("mfi_device_error: the flag could not be read")
    return v


def check_device(what: str) -> None:
    """Raise MfiDeviceError (and clear the flag) if a kernel reported a failure."""
    v = device_error(clear=True)
    if v:
        raise MfiDeviceError(f"{what}: device error {v}: {DEVICE_ERRORS.get(v, 'unknown code')}")


def load():
    """Load (once) and return the ctypes handle; raise if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m moe_fused_inference_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().mfi_last_error().decode(errors="replace")
        raise MfiError(f"{what}: {msg} (status {status})")
    if _CHECK_DEVICE:
        check_device(what)
