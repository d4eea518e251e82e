"""ZTCP cold-page codec for NVIDIA B200 (sm_100a).

Modules:
  capi           -- ctypes binding of the C-ABI (include/ztcp_b200.h), loads libztcp_b200.so
  codec          -- GPU-native batch API: block tables, per-page metadata, stream-ordered
  fused_ext      -- drop-in for the reference's native module (NativeCppFusedColdPageCodec._ext)
  cold_page_spec -- wire-format spec mirror (header, presets, geometry, payload sizes)
  build          -- nvcc build recipe for libztcp_b200.so
"""
from . import build, capi, cold_page_spec  # noqa: F401

__all__ = ["build", "capi", "cold_page_spec", "codec", "fused_ext"]
