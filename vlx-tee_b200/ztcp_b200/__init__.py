"""ZTCP cold-page codec for NVIDIA B200 (sm_100a).

Modules:
  capi           -- ctypes binding of the C-ABI (include/ztcp_b200.h), loads libztcp_b200.so
  codec          -- GPU-native batch API: block tables, per-page metadata, stream-ordered
  fused_ext      -- drop-in for the reference's native module (NativeCppFusedColdPageCodec._ext)
  cold_page_spec -- wire-format spec mirror (header, presets, geometry, payload sizes)
  session        -- GPU-native session codec: the reference wrapper's six methods on CUDA tensors
  offload        -- egress to / ingress from pinned host memory with copies overlapped across slots
  hooks          -- engine offload hooks: pinned staging ring, page codec with a per-page recompute fallback
  keyring        -- session keyring with the reference's interface, per-page tables in the C++ ledger
  ledger         -- ctypes binding of the ledger C-ABI (include/ztcp_ledger.h)
  errors         -- exception classes with the reference's names and hierarchy
  sharding       -- page partitioning over GPUs and the max-over-ranks timing reduction
  workload       -- seeded synthetic KV pages and session material of the benchmark configurations
  build          -- nvcc build recipe for libztcp_b200.so
"""
from . import build, capi, cold_page_spec  # noqa: F401

__all__ = ["build", "capi", "cold_page_spec", "codec", "errors", "fused_ext", "hooks", "keyring", "ledger", "offload",
           "session", "sharding", "workload"]
