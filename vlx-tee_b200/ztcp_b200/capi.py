"""ctypes binding of the C-ABI in include/ztcp_b200.h.

This module loads the in-tree ``libztcp_b200.so`` and fails loudly when it is
missing: there is no CPU fallback anywhere in the product path.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

ZTCP_OK = 0
ZTCP_EINVAL = -1
ZTCP_ECUDA = -2
DTYPE_F16 = 0
DTYPE_BF16 = 1

PAGE_OK = 0
PAGE_BAD_MAGIC = 1
PAGE_AAD_MISMATCH = 2
PAGE_MAC_FAILED = 3
PAGE_BAD_FLAGS = 4
PAGE_TRUNCATED = 5
PAGE_BAD_BLOCK = 6

# every symbol include/ztcp_b200.h declares
EXPORTED_SYMBOLS = (
    "ztcp_last_error",
    "ztcp_version",
    "ztcp_min_payload_bytes",
    "ztcp_spec_payload_bytes",
    "ztcp_encode_pages",
    "ztcp_decode_pages",
    "ztcp_verify_pages",
    "ztcp_chacha20_xor",
    "ztcp_siphash24_128",
    "ztcp_gather",
    "ztcp_decode_pages_noalloc",
)
# every symbol include/ztcp_measure.h declares (measurement entry points, not part of the drop-in boundary)
MEASURE_SYMBOLS = ("ztcp_measure_int_peaks", "ztcp_mark_phase")
MEASURE_SCRATCH_BYTES = 8 << 20  # ZTCP_MEASURE_SCRATCH_BYTES


class Geometry(C.Structure):
    _fields_ = [
        ("num_tokens", C.c_int64),
        ("num_heads", C.c_int64),
        ("head_dim", C.c_int64),
        ("rope_dim", C.c_int64),
        ("is_mla_single_buffer", C.c_int32),
        ("reserved", C.c_int32),
    ]


class Keys(C.Structure):
    _fields_ = [("enc", C.c_uint64 * 4), ("mac", C.c_uint64 * 2)]


class PageBatch(C.Structure):
    _fields_ = [
        ("n_pages", C.c_int64),
        ("kv_block", C.c_void_p),
        ("token_hash", C.c_void_p),
        ("sequence_nonce", C.c_void_p),
        ("layer_id", C.c_void_p),
        ("base_sequence_nonce", C.c_uint64),
        ("tenant_id_hash", C.c_uint32),
        ("model_id_hash", C.c_uint32),
        ("layer_id_uniform", C.c_uint16),
        ("head_group_id", C.c_uint16),
        ("options", C.c_int32),
        ("kv_pool_pages", C.c_int64),
    ]


class IntPeaks(C.Structure):
    _fields_ = [
        ("chacha20_blocks_per_s", C.c_double),
        ("sip_words_per_s", C.c_double),
        ("sip_chain_cycles_per_word", C.c_double),
        ("sip_chain_ms", C.c_double),
        ("sms", C.c_int32),
        ("reserved", C.c_int32),
    ]


OPT_NEON_ARITH = 1
OPT_PAGE_FALLBACK = 2
NOALLOC_MAX_PAGES = 65536  # ZTCP_NOALLOC_MAX_PAGES


class ZtcpError(RuntimeError):
    """A C-ABI call rejected its arguments or failed to launch."""


_lib = None


def library_path() -> str:
    return _build.LIB_PATH


def load() -> C.CDLL:
    """Load libztcp_b200.so (built in-tree by build.py); raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not os.path.isfile(path):
        raise ImportError(
            f"{path} is missing: build it with `python vlx-tee_b200/ztcp_b200/build.py` "
            "(the ZTCP codec has no CPU fallback)"
        )
    L = C.CDLL(path)
    vp, i32, i64, u32, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint32, C.c_uint64
    L.ztcp_last_error.restype = C.c_char_p
    L.ztcp_last_error.argtypes = []
    L.ztcp_version.restype = i32
    L.ztcp_version.argtypes = []
    L.ztcp_min_payload_bytes.restype = i64
    L.ztcp_min_payload_bytes.argtypes = [i32, i32, C.POINTER(Geometry), i32]
    L.ztcp_spec_payload_bytes.restype = i64
    L.ztcp_spec_payload_bytes.argtypes = [i32, i32, C.POINTER(Geometry), i32]
    L.ztcp_encode_pages.restype = i32
    L.ztcp_encode_pages.argtypes = [vp, vp, i32, C.POINTER(Geometry), C.POINTER(PageBatch), i32, i32, i64,
                                    C.POINTER(Keys), vp, vp]
    L.ztcp_decode_pages.restype = i32
    L.ztcp_decode_pages.argtypes = [vp, i64, C.POINTER(Geometry), C.POINTER(PageBatch), C.POINTER(Keys), vp, vp,
                                    vp, vp, vp]
    L.ztcp_verify_pages.restype = i32
    L.ztcp_verify_pages.argtypes = [vp, i64, C.POINTER(Geometry), C.POINTER(PageBatch), C.POINTER(Keys), vp, vp, vp]
    L.ztcp_chacha20_xor.restype = i32
    L.ztcp_chacha20_xor.argtypes = [vp, vp, i64, C.c_char_p, u32, C.c_char_p, vp]
    L.ztcp_siphash24_128.restype = i32
    L.ztcp_siphash24_128.argtypes = [vp, i64, u64, u64, vp, vp]
    L.ztcp_decode_pages_noalloc.restype = i32
    L.ztcp_decode_pages_noalloc.argtypes = [vp, i64, C.POINTER(Geometry), C.POINTER(PageBatch), C.POINTER(Keys), vp,
                                            vp, vp, vp]
    L.ztcp_measure_int_peaks.restype = i32
    L.ztcp_measure_int_peaks.argtypes = [vp, i64, C.POINTER(IntPeaks)]
    L.ztcp_mark_phase.restype = i32
    L.ztcp_mark_phase.argtypes = [vp]
    L.ztcp_gather.restype = i32
    L.ztcp_gather.argtypes = [vp, i32, C.POINTER(vp), C.POINTER(i32), C.POINTER(i64), i32, vp]
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != ZTCP_OK:
        msg = load().ztcp_last_error().decode("utf-8", "replace")
        raise ZtcpError(msg)


def geometry(num_tokens: int, num_heads: int, head_dim: int, rope_dim: int, is_mla: bool) -> Geometry:
    return Geometry(num_tokens, num_heads, head_dim, rope_dim, 1 if is_mla else 0, 0)


def keys(k0: int, k1: int, k2: int, k3: int, mk0: int, mk1: int) -> Keys:
    m = (1 << 64) - 1
    k = Keys()
    for i, v in enumerate((k0, k1, k2, k3)):
        k.enc[i] = int(v) & m
    k.mac[0] = int(mk0) & m
    k.mac[1] = int(mk1) & m
    return k
