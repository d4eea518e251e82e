"""C-ABI library on a CPU-only host: it loads, exports every declared symbol, sizes payloads like the
spec, and rejects invalid arguments with the reference's messages before touching the GPU."""
from __future__ import annotations

import ctypes as C
import os
import re

import pytest

from ztcp_b200 import build, capi
from ztcp_b200.cold_page_spec import ColdPageAAD, ColdPageGeometry, QuantPreset, RoPEMode

INCLUDE = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
HEADER = os.path.join(INCLUDE, "ztcp_b200.h")
LEDGER_HEADER = os.path.join(INCLUDE, "ztcp_ledger.h")
MEASURE_HEADER = os.path.join(INCLUDE, "ztcp_measure.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return capi.load()


def declared_functions(path=HEADER):
    text = open(path).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(ztcp_\w+)\(", text, re.M)))


def test_exports_every_declared_symbol(lib):
    from ztcp_b200 import ledger

    names = declared_functions()
    assert set(names) == set(capi.EXPORTED_SYMBOLS)
    ledger_names = declared_functions(LEDGER_HEADER)
    assert set(ledger_names) == set(ledger.LEDGER_SYMBOLS)
    measure_names = declared_functions(MEASURE_HEADER)
    assert set(measure_names) == set(capi.MEASURE_SYMBOLS)
    for n in names + ledger_names + measure_names:
        assert hasattr(lib, n), n
    assert lib.ztcp_version() >= 100


@pytest.mark.parametrize("geo", [ColdPageGeometry(), ColdPageGeometry(64, 1, 576, 64, is_mla_single_buffer=True),
                                 ColdPageGeometry(3, 1, 16, 0), ColdPageGeometry(5, 3, 48, 48),
                                 ColdPageGeometry(1, 1, 16, 16)])
def test_payload_sizes(lib, oracle, geo):
    for p in QuantPreset:
        for r in RoPEMode:
            g = capi.geometry(geo.num_tokens, geo.num_kv_heads, geo.head_dim, geo.rope_dim, geo.is_mla_single_buffer)
            has_v = 0 if geo.is_mla_single_buffer else 1
            spec = lib.ztcp_spec_payload_bytes(int(p), int(r), C.byref(g), has_v)
            assert spec == geo.payload_bytes(p, r)
            assert lib.ztcp_min_payload_bytes(int(p), int(r), C.byref(g), has_v) == geo.min_payload_bytes(p, r)
            assert spec == oracle.spec_payload_bytes(p, r, geo.vectors_per_buffer, geo.head_dim, geo.rope_dim,
                                                     has_v)
    g = capi.geometry(64, 8, 128, 64, False)
    assert lib.ztcp_spec_payload_bytes(0, 1, C.byref(g), 1) == -1
    assert lib.ztcp_spec_payload_bytes(1, 3, C.byref(g), 1) == -1


def test_header_pack_roundtrip():
    aad = ColdPageAAD(0xDEADBEEF, 0x01020304, 0xABCD, 2**64 - 3, 2**63 + 5, QuantPreset.INT4_SYM,
                      RoPEMode.PRESERVE_FP8, 0x0102)
    raw = aad.pack_header()
    assert len(raw) == 32 and raw[:4] == bytes([0x54, 0x5A, 1, 0x11])
    assert ColdPageAAD.unpack_header(raw) == aad


FAKE = 0x10000  # never dereferenced: validation fails before any device access


def _encode(lib, **kw):
    a = dict(k=FAKE, v=FAKE, dtype=capi.DTYPE_F16, geom=capi.geometry(64, 8, 128, 64, False), n=4, preset=1,
             rope_mode=1, exp=98304, out=FAKE, token=FAKE)
    a.update(kw)
    b = capi.PageBatch()
    b.n_pages = a["n"]
    b.token_hash = a["token"]
    b.options = a.get("options", 0)
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    rc = lib.ztcp_encode_pages(a["k"], a["v"], a["dtype"], C.byref(a["geom"]), C.byref(b), a["preset"],
                               a["rope_mode"], a["exp"], C.byref(keys), a["out"], None)
    return rc, lib.ztcp_last_error().decode()


@pytest.mark.parametrize("kw,msg", [
    (dict(preset=0), "Invalid preset (must be 1..3)"),
    (dict(preset=4), "Invalid preset (must be 1..3)"),
    (dict(rope_mode=3), "Invalid rope_mode (must be 0..2)"),
    (dict(exp=98300), "expected_payload_bytes smaller than required payload"),
    (dict(geom=capi.geometry(64, 8, 120, 64, False)), "Invalid k_pages dimensions"),
    (dict(geom=capi.geometry(0, 8, 128, 64, False)), "Invalid k_pages dimensions"),
    (dict(geom=capi.geometry(64, 8, 128, 72, False)), "Invalid rope_dim"),
    (dict(geom=capi.geometry(64, 8, 128, 144, False)), "Invalid rope_dim"),
    (dict(n=0), "batch must hold at least one page"),
    (dict(token=None), "page_token_hashes must not be NULL"),
    (dict(k=FAKE + 8), "k_pages / v_pages must be 16-byte aligned"),
    (dict(dtype=7), "k_pages must be float16 or bfloat16"),
    (dict(options=4), "unknown page batch options"),
    (dict(options=capi.OPT_NEON_ARITH | 8), "unknown page batch options"),
])
def test_encode_validation(lib, kw, msg):
    rc, err = _encode(lib, **kw)
    assert rc == capi.ZTCP_EINVAL
    assert err == msg


def test_decode_validation(lib):
    b = capi.PageBatch()
    b.n_pages = 2
    b.token_hash = FAKE
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    g = capi.geometry(64, 8, 128, 64, False)
    rc = lib.ztcp_decode_pages(FAKE, 48, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error() == b"cold_blob too small"
    rc = lib.ztcp_decode_pages(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, None, FAKE, FAKE, None)
    assert lib.ztcp_last_error() == b"out_v_pages is required for non-MLA geometry"
    gm = capi.geometry(64, 1, 576, 64, True)
    rc = lib.ztcp_decode_pages(FAKE, 25136, C.byref(gm), C.byref(b), C.byref(keys), FAKE, FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and b"must be NULL" in lib.ztcp_last_error()


def test_kat_validation(lib):
    assert lib.ztcp_chacha20_xor(FAKE, FAKE, -1, b"\0" * 32, 0, b"\0" * 12, None) == capi.ZTCP_EINVAL
    assert lib.ztcp_siphash24_128(FAKE, 8, 1, 2, None, None) == capi.ZTCP_EINVAL


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(capi, "_lib", None)
    monkeypatch.setattr(capi, "library_path", lambda: str(tmp_path / "absent.so"))
    with pytest.raises(ImportError, match="no CPU fallback"):
        capi.load()


def test_decode_rejects_unknown_options(lib):
    b = capi.PageBatch()
    b.n_pages = 2
    b.token_hash = FAKE
    b.options = capi.OPT_PAGE_FALLBACK | 16
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    g = capi.geometry(64, 8, 128, 64, False)
    rc = lib.ztcp_decode_pages(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error() == b"unknown page batch options"


def test_noalloc_decode_validation(lib):
    """The no-allocation decode rejects a missing batch, a missing fail flag and batches beyond its fixed
    buffer before it touches a GPU."""
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    g = capi.geometry(64, 8, 128, 64, False)
    rc = lib.ztcp_decode_pages_noalloc(FAKE, 98352, C.byref(g), None, C.byref(keys), FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error() == b"page batch must not be NULL"
    b = capi.PageBatch()
    b.n_pages = 2
    b.token_hash = FAKE
    rc = lib.ztcp_decode_pages_noalloc(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, None, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error() == b"any_fail must not be NULL"
    b.n_pages = capi.NOALLOC_MAX_PAGES + 1
    rc = lib.ztcp_decode_pages_noalloc(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL
    assert lib.ztcp_last_error() == b"batch of 65537 pages exceeds the no-allocation decode's limit of 65536 pages per call"


def test_pool_size_validation(lib):
    """A block table needs the pool size its entries are checked against on the device; without a table a
    given pool size must hold the batch."""
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    g = capi.geometry(64, 8, 128, 64, False)
    b = capi.PageBatch()
    b.n_pages = 4
    b.token_hash = FAKE
    b.kv_block = FAKE
    rc = lib.ztcp_decode_pages(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error().startswith(b"kv_pool_pages is required")
    rc = lib.ztcp_encode_pages(FAKE, FAKE, 1, C.byref(g), C.byref(b), 1, 1, 98304, C.byref(keys), FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error().startswith(b"kv_pool_pages is required")
    b.kv_pool_pages = -1
    rc = lib.ztcp_verify_pages(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error() == b"kv_pool_pages must be non-negative"
    b.kv_block = None
    b.kv_pool_pages = 3
    rc = lib.ztcp_decode_pages(FAKE, 98352, C.byref(g), C.byref(b), C.byref(keys), FAKE, FAKE, FAKE, FAKE, None)
    assert rc == capi.ZTCP_EINVAL and lib.ztcp_last_error() == b"batch has more pages than kv_pool_pages"


def test_measurement_entry_points_validate(lib):
    out = capi.IntPeaks()
    assert lib.ztcp_measure_int_peaks(None, capi.MEASURE_SCRATCH_BYTES, C.byref(out)) == capi.ZTCP_EINVAL
    assert lib.ztcp_last_error() == b"scratch and out must not be NULL"
    assert lib.ztcp_measure_int_peaks(FAKE + 4, capi.MEASURE_SCRATCH_BYTES, C.byref(out)) == capi.ZTCP_EINVAL
    assert lib.ztcp_mark_phase(None) == capi.ZTCP_OK
