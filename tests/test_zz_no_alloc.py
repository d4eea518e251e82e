"""ztcp_decode_pages_noalloc -- decode for callers that cannot allocate device memory on the decode path
(an engine that gives all device memory to its KV pool at start-up, or a plugin that only sees the
engine's buffers).  Called through the C-ABI, it must give the same K/V bytes and the same batch verdict
as ztcp_decode_pages with caller-provided status buffers, call after call (it reuses one status buffer
inside the library), and refuse batches larger than its fixed buffer.

This file is collected last so that a run stopping at its first failure has run every other test."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _batch(n, seed, tamper_page=None):
    from ztcp_b200 import capi, codec, workload

    m = workload.session_material(seed)
    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=seed)
    k = torch.from_numpy(k32).to(torch.bfloat16).to(DEV)
    v = torch.from_numpy(v32).to(torch.bfloat16).to(DEV)
    toks = torch.from_numpy(workload.token_hashes(n, seed + 1).view(np.int64)).to(DEV)
    keys = capi.keys(*m["key"], *m["mac_key"])
    blobs = torch.empty((n, 98352), dtype=torch.uint8, device=DEV)
    codec.encode_pages(k, v, toks, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                       head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
    if tamper_page is not None:
        blobs[tamper_page, 7000] ^= 0x10
    return m, toks, keys, blobs


def _decode_both(lib, m, toks, keys, blobs, page_fallback=False):
    from ztcp_b200 import capi, codec

    n = blobs.shape[0]
    # the existing entry point, with its status buffers from the caller
    ko_ref = torch.full((n, 64, 8, 128), 5.0, dtype=torch.float16, device=DEV)
    vo_ref = torch.full_like(ko_ref, 5.0)
    _, fail_ref = codec.decode_pages(blobs, toks, ko_ref, vo_ref, rope_dim=64, is_mla=False,
                                     tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                     keys=keys, page_fallback=page_fallback)
    # the no-allocation entry point through the C-ABI: only inputs, outputs and the fail flag
    ko = torch.full_like(ko_ref, 9.0)
    vo = torch.full_like(ko_ref, 9.0)
    fail = torch.full((1,), 7, dtype=torch.int32, device=DEV)
    geom = capi.geometry(64, 8, 128, 64, False)
    batch = codec._page_batch(n, toks, None, None, None, 0, m["tenant"], m["model"], m["layer"], 0,
                              capi.OPT_PAGE_FALLBACK if page_fallback else 0)
    rc = lib.ztcp_decode_pages_noalloc(blobs.data_ptr(), blobs.shape[1], C.byref(geom), C.byref(batch),
                                       C.byref(keys), ko.data_ptr(), vo.data_ptr(), fail.data_ptr(),
                                       torch.cuda.current_stream(DEV).cuda_stream)
    capi.check(rc)
    torch.cuda.synchronize()
    return (ko_ref, vo_ref, int(fail_ref.item())), (ko, vo, int(fail.item()))


def test_noalloc_decode_equals_decode_pages_call_after_call():
    from ztcp_b200 import build, capi

    build.build()
    lib = capi.load()
    # two calls in a row: a clean batch, then a batch with a tampered page (all outputs zeroed), then the
    # clean batch again -- the shared status buffer must not carry one call's verdicts into the next
    cases = [_batch(8, 301), _batch(5, 302, tamper_page=3)]
    cases.append(cases[0])
    expect_fail = [0, 1, 0]
    for (m, toks, keys, blobs), want_fail in zip(cases, expect_fail):
        (ko_ref, vo_ref, f_ref), (ko, vo, f) = _decode_both(lib, m, toks, keys, blobs)
        assert f_ref == want_fail and f == want_fail
        assert torch.equal(ko.view(torch.int16), ko_ref.view(torch.int16))
        assert torch.equal(vo.view(torch.int16), vo_ref.view(torch.int16))
        if want_fail:
            assert not ko.any() and not vo.any()


def test_noalloc_page_fallback_reads_this_calls_verdicts():
    """With the per-page fallback the decrypt pass reads the library's status array page by page: a tampered
    batch zeroes only its failing page, and a following clean batch of as many or fewer pages zeroes none --
    no verdict of one call leaks into the next."""
    from ztcp_b200 import build, capi

    build.build()
    lib = capi.load()
    tampered = _batch(6, 311, tamper_page=2)
    clean_same = _batch(6, 312)
    clean_fewer = _batch(4, 313)
    for case, bad_page in ((tampered, 2), (clean_same, None), (clean_fewer, None), (tampered, 2)):
        m, toks, keys, blobs = case
        (ko_ref, vo_ref, f_ref), (ko, vo, f) = _decode_both(lib, m, toks, keys, blobs, page_fallback=True)
        assert f_ref == f == (1 if bad_page is not None else 0)
        assert torch.equal(ko.view(torch.int16), ko_ref.view(torch.int16))
        assert torch.equal(vo.view(torch.int16), vo_ref.view(torch.int16))
        for p in range(blobs.shape[0]):
            zeroed = not ko[p].any() and not vo[p].any()
            assert zeroed == (p == bad_page), p


def test_noalloc_decode_rejects_batches_beyond_its_buffer():
    from ztcp_b200 import build, capi, codec

    build.build()
    lib = capi.load()
    n = capi.NOALLOC_MAX_PAGES + 1
    toks = torch.zeros(1, dtype=torch.int64, device=DEV)
    batch = codec._page_batch(n, toks, None, None, None, 0, 1, 2, 3, 0)
    geom = capi.geometry(64, 8, 128, 64, False)
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    fail = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.ztcp_decode_pages_noalloc(None, 98352, C.byref(geom), C.byref(batch), C.byref(keys), None, None,
                                       fail.data_ptr(), None)
    assert rc == capi.ZTCP_EINVAL
    assert b"limit of 65536 pages" in lib.ztcp_last_error()
