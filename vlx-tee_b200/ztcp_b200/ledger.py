"""ctypes binding of the keyring ledger (include/ztcp_ledger.h) in libztcp_b200.so.

The ledger holds, per session, the burned 96-bit ChaCha20 nonces, the per-slot freshness watermarks and
the session's largest sequence nonce, and checks whole batches in C++ (all-or-nothing).  Host code only:
it needs the built library but no GPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import capi

OK = 0
ESTALE = -1
EREUSE = -2
ENOSESSION = -3
EINVAL = -4
EMISMATCH = -5

# every symbol include/ztcp_ledger.h declares
LEDGER_SYMBOLS = (
    "ztcp_ledger_create", "ztcp_ledger_destroy", "ztcp_ledger_open", "ztcp_ledger_close", "ztcp_ledger_is_open",
    "ztcp_ledger_next_nonce", "ztcp_ledger_max_nonce", "ztcp_ledger_preflight", "ztcp_reservation_last_seq",
    "ztcp_reservation_pages", "ztcp_ledger_commit", "ztcp_reservation_free", "ztcp_ledger_freshness_batch",
    "ztcp_ledger_freshness_one", "ztcp_ledger_parse_headers",
)


class Error(C.Structure):
    _fields_ = [("code", C.c_int32), ("kind", C.c_int32), ("index", C.c_int64), ("seq", C.c_uint64),
                ("ref", C.c_uint64), ("loc", C.c_uint32), ("reserved", C.c_uint32)]


class FreshRecord(C.Structure):
    _fields_ = [("model_id_hash", C.c_uint32), ("layer_id", C.c_uint16), ("head_group_id", C.c_uint16),
                ("page_token_hash", C.c_uint64), ("sequence_nonce", C.c_uint64)]


# numpy view of an array of FreshRecord
RECORD_DTYPE = np.dtype([("model_id_hash", "<u4"), ("layer_id", "<u2"), ("head_group_id", "<u2"),
                         ("page_token_hash", "<u8"), ("sequence_nonce", "<u8")])
assert RECORD_DTYPE.itemsize == C.sizeof(FreshRecord)

_bound = None


def _lib() -> C.CDLL:
    global _bound
    L = capi.load()
    if _bound is L:
        return L
    vp, i32, i64, u16, u32, u64 = C.c_void_p, C.c_int32, C.c_int64, C.c_uint16, C.c_uint32, C.c_uint64
    L.ztcp_ledger_create.restype = vp
    L.ztcp_ledger_create.argtypes = []
    L.ztcp_ledger_destroy.restype = None
    L.ztcp_ledger_destroy.argtypes = [vp]
    for name in ("ztcp_ledger_open", "ztcp_ledger_close", "ztcp_ledger_is_open"):
        getattr(L, name).restype = i32
        getattr(L, name).argtypes = [vp, u64]
    L.ztcp_ledger_next_nonce.restype = i32
    L.ztcp_ledger_next_nonce.argtypes = [vp, u64, u64, C.POINTER(u64), C.POINTER(u64)]
    L.ztcp_ledger_max_nonce.restype = i32
    L.ztcp_ledger_max_nonce.argtypes = [vp, u64, C.POINTER(u64), C.POINTER(u64)]
    L.ztcp_ledger_preflight.restype = i32
    L.ztcp_ledger_preflight.argtypes = [vp, u64, u32, u16, u16, u64, vp, i64, C.POINTER(vp), C.POINTER(Error)]
    L.ztcp_reservation_last_seq.restype = u64
    L.ztcp_reservation_last_seq.argtypes = [vp]
    L.ztcp_reservation_pages.restype = i64
    L.ztcp_reservation_pages.argtypes = [vp]
    L.ztcp_ledger_commit.restype = i32
    L.ztcp_ledger_commit.argtypes = [vp, u64, vp]
    L.ztcp_reservation_free.restype = None
    L.ztcp_reservation_free.argtypes = [vp]
    L.ztcp_ledger_freshness_batch.restype = i32
    L.ztcp_ledger_freshness_batch.argtypes = [vp, u64, vp, i64, i32, u64, C.POINTER(Error)]
    L.ztcp_ledger_freshness_one.restype = i32
    L.ztcp_ledger_freshness_one.argtypes = [vp, u64, C.POINTER(FreshRecord), i32, u64, i32, u64, C.POINTER(Error)]
    L.ztcp_ledger_parse_headers.restype = i32
    L.ztcp_ledger_parse_headers.argtypes = [vp, i64, i64, vp]
    _bound = L
    return L


class LedgerError(Exception):
    """A failed ledger check; `err` is the ztcp_ledger_error the library filled in."""

    def __init__(self, code: int, err: Error):
        super().__init__(code)
        self.code = code
        self.err = err


class Reservation:
    """Staged slot watermarks of one preflight (owns the C handle until freed)."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)

    @property
    def handle(self) -> C.c_void_p:
        if not self._h:
            raise RuntimeError("reservation already freed")
        return self._h

    @property
    def last_seq(self) -> int:
        return int(_lib().ztcp_reservation_last_seq(self.handle))

    @property
    def pages(self) -> int:
        return int(_lib().ztcp_reservation_pages(self.handle))

    def free(self) -> None:
        if self._h:
            _lib().ztcp_reservation_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Ledger:
    def __init__(self):
        self._L = _lib()
        self._p = C.c_void_p(self._L.ztcp_ledger_create())
        if not self._p:
            raise MemoryError("ztcp_ledger_create failed")

    def __del__(self):
        try:
            if self._p:
                self._L.ztcp_ledger_destroy(self._p)
                self._p = C.c_void_p()
        except Exception:
            pass

    def _check(self, rc: int, err: Error | None = None) -> None:
        if rc == OK:
            return
        if rc in (ESTALE, EREUSE, EMISMATCH):
            raise LedgerError(rc, err)
        raise RuntimeError(f"ztcp ledger call failed with code {rc}")

    def open(self, session: int) -> None:
        self._check(self._L.ztcp_ledger_open(self._p, session))

    def close(self, session: int) -> bool:
        return bool(self._L.ztcp_ledger_close(self._p, session))

    def is_open(self, session: int) -> bool:
        return bool(self._L.ztcp_ledger_is_open(self._p, session))

    def next_nonce(self, session: int, count: int) -> int:
        lo, hi = C.c_uint64(), C.c_uint64()
        self._check(self._L.ztcp_ledger_next_nonce(self._p, session, count, C.byref(lo), C.byref(hi)))
        return (int(hi.value) << 64) | int(lo.value)

    def max_nonce(self, session: int) -> int:
        lo, hi = C.c_uint64(), C.c_uint64()
        self._check(self._L.ztcp_ledger_max_nonce(self._p, session, C.byref(lo), C.byref(hi)))
        return (int(hi.value) << 64) | int(lo.value)

    def preflight(self, session: int, model_id_hash: int, layer_id: int, head_group_id: int, base_seq: int,
                  token_hashes) -> Reservation:
        toks = np.ascontiguousarray(np.asarray(token_hashes, dtype=np.uint64) if not isinstance(token_hashes, list)
                                    else np.array([t & 0xFFFFFFFFFFFFFFFF for t in token_hashes], dtype=np.uint64))
        out, err = C.c_void_p(), Error()
        rc = self._L.ztcp_ledger_preflight(self._p, session, model_id_hash, layer_id, head_group_id, base_seq,
                                           toks.ctypes.data, toks.size, C.byref(out), C.byref(err))
        self._check(rc, err)
        return Reservation(out.value)

    def commit(self, session: int, r: Reservation) -> None:
        self._check(self._L.ztcp_ledger_commit(self._p, session, r.handle))

    def freshness_batch(self, session: int, records: np.ndarray, min_seq: int | None) -> None:
        rec = np.ascontiguousarray(records, dtype=RECORD_DTYPE)
        err = Error()
        rc = self._L.ztcp_ledger_freshness_batch(self._p, session, rec.ctypes.data if rec.size else None, rec.size,
                                                 int(min_seq is not None), 0 if min_seq is None else min_seq,
                                                 C.byref(err))
        self._check(rc, err)

    def freshness_one(self, session: int, record: FreshRecord, min_seq: int | None, expected: int | None) -> None:
        err = Error()
        rc = self._L.ztcp_ledger_freshness_one(self._p, session, C.byref(record), int(min_seq is not None),
                                               0 if min_seq is None else min_seq, int(expected is not None),
                                               0 if expected is None else expected, C.byref(err))
        self._check(rc, err)


def records_from_tuples(records) -> np.ndarray:
    """(model_id_hash, layer_id, head_group_id, page_token_hash, sequence_nonce) tuples -> record array."""
    out = np.empty(len(records), dtype=RECORD_DTYPE)
    if len(records):
        cols = list(zip(*records))
        out["model_id_hash"] = np.array([x & 0xFFFFFFFF for x in cols[0]], dtype=np.uint64).astype(np.uint32)
        out["layer_id"] = np.array([x & 0xFFFF for x in cols[1]], dtype=np.uint32).astype(np.uint16)
        out["head_group_id"] = np.array([x & 0xFFFF for x in cols[2]], dtype=np.uint32).astype(np.uint16)
        out["page_token_hash"] = np.array([x & 0xFFFFFFFFFFFFFFFF for x in cols[3]], dtype=np.uint64)
        out["sequence_nonce"] = np.array([x & 0xFFFFFFFFFFFFFFFF for x in cols[4]], dtype=np.uint64)
    return out


def records_from_headers(blobs_u8: np.ndarray) -> np.ndarray:
    """Freshness records of every row of a [n, >=32] uint8 array of blobs (or headers), parsed in C++."""
    a = np.ascontiguousarray(blobs_u8, dtype=np.uint8)
    if a.ndim != 2 or a.shape[1] < 32:
        raise RuntimeError("blobs must be a [n, >= 32] uint8 array")
    out = np.empty(a.shape[0], dtype=RECORD_DTYPE)
    rc = _lib().ztcp_ledger_parse_headers(a.ctypes.data if a.size else None, a.shape[1], a.shape[0],
                                          out.ctypes.data if out.size else None)
    if rc != OK:
        raise RuntimeError(f"ztcp_ledger_parse_headers failed with code {rc}")
    return out
