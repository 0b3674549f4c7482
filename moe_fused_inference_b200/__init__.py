"""B200-native (sm_100a) MXFP4 grouped-MoE expert path.

Public surface:
  fp4_ext.get_ext() / fp4_ext.get_decode_ext()  drop-in for the reference's
                                               runtime/fp4_ext.py operators
  layer.MoELayer                               device-routed fused MoE layer
  layer.quantize_rows                          GPU quantize_expert_tensor
The compute lives in libmoe_fp4.so (C ABI: include/moe_fp4.h).
"""

from . import fp4_ext  # noqa: F401

__all__ = ["fp4_ext"]
