"""Prepared codec calls (codec.prepare_encode / prepare_decode): checked and packed once, enqueued many times
on any stream.  Every call must read the tensors' current contents (new K/V, tampered or restored blobs),
write the same bytes as a one-shot call and as the oracle, keep its own copy of the keys, and hand back the
same status / any_fail tensors."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
PAGES = 24


def _material():
    from ztcp_b200 import capi, workload

    m = workload.session_material(301)
    return m, capi.keys(*m["key"], *m["mac_key"])


def _encode_kw(m, keys):
    return dict(rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304, tenant_id_hash=m["tenant"],
                model_id_hash=m["model"], layer_id=m["layer"], head_group_id=m["head_group"],
                base_sequence_nonce=m["base_seq"], keys=keys)


def _decode_kw(m, keys):
    return dict(rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                keys=keys)


def test_prepared_encode_reads_current_inputs(oracle):
    from ztcp_b200 import codec, workload

    m, keys = _material()
    k, v = workload.kv_pages_torch(PAGES, workload.GQA, seed=302, dtype=torch.float16, device=DEV)
    toks_np = workload.token_hashes(PAGES, 303)
    toks = torch.from_numpy(toks_np).to(DEV)
    blobs = torch.full((PAGES, 98352), 0x77, dtype=torch.uint8, device=DEV)
    call = codec.prepare_encode(k, v, toks, blobs, **_encode_kw(m, keys))
    keys.enc[0] ^= 0xFFFF  # the caller reuses its key block: the prepared call kept its own copy
    keys.mac[1] = 0
    _, keys_ref = _material()

    side = torch.cuda.Stream(device=DEV)
    call(side)  # a torch stream
    side.synchronize()
    once = torch.empty_like(blobs)
    codec.encode_pages(k, v, toks, once, **_encode_kw(m, keys_ref))
    torch.cuda.synchronize()
    assert torch.equal(blobs, once)

    # new K/V in place, same addresses: the next call encodes them (raw stream handle this time)
    k2, v2 = workload.kv_pages_torch(PAGES, workload.GQA, seed=304, dtype=torch.float16, device=DEV)
    k.copy_(k2)
    v.copy_(v2)
    torch.cuda.synchronize()
    call(torch.cuda.current_stream(DEV).cuda_stream)
    torch.cuda.synchronize()
    want = helpers.oracle_encode(oracle, k.cpu().numpy(), v.cpu().numpy(), toks_np, 64, 1, 1, 98304, m)
    np.testing.assert_array_equal(blobs.cpu().numpy(), want)


def test_prepared_decode_sees_tamper_and_restore():
    from ztcp_b200 import capi, codec, workload

    m, keys = _material()
    k, v = workload.kv_pages_torch(PAGES, workload.GQA, seed=305, dtype=torch.float16, device=DEV)
    toks = torch.from_numpy(workload.token_hashes(PAGES, 306)).to(DEV)
    blobs = torch.empty((PAGES, 98352), dtype=torch.uint8, device=DEV)
    codec.encode_pages(k, v, toks, blobs, **_encode_kw(m, keys))
    ko, vo = torch.empty_like(k), torch.empty_like(v)
    call = codec.prepare_decode(blobs, toks, ko, vo, **_decode_kw(m, keys))
    st, fail = call()
    torch.cuda.synchronize()
    assert int(fail.item()) == 0 and not st.any()
    ref_k, ref_v = ko.clone(), vo.clone()
    st_once, _ = codec.decode_pages(blobs, toks, torch.empty_like(k), torch.empty_like(v), **_decode_kw(m, keys))
    torch.cuda.synchronize()
    assert not st_once.any()

    saved = blobs[7, 5000].item()
    blobs[7, 5000] ^= 0x10                   # one payload byte of page 7
    st2, fail2 = call(torch.cuda.Stream(device=DEV))
    torch.cuda.synchronize()
    assert st2 is st and fail2 is fail       # the same device outputs at every call
    assert int(fail.item()) == 1 and int(st[7]) == capi.PAGE_MAC_FAILED and int(st.ne(0).sum()) == 1
    assert not ko.any() and not vo.any()     # all-or-nothing: every page zeroed

    blobs[7, 5000] = saved
    call()
    torch.cuda.synchronize()
    assert int(fail.item()) == 0 and not st.any()
    assert torch.equal(ko, ref_k) and torch.equal(vo, ref_v)


def test_prepared_call_rejects_bad_arguments_once():
    from ztcp_b200 import capi, codec, workload

    m, keys = _material()
    k, v = workload.kv_pages_torch(4, workload.GQA, seed=307, dtype=torch.float16, device=DEV)
    toks = torch.from_numpy(workload.token_hashes(4, 308)).to(DEV)
    blobs = torch.full((4, 98352), 0x77, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="out_blobs shape"):
        codec.prepare_encode(k, v, toks, blobs.view(-1)[:4 * 98351].view(4, 98351), **_encode_kw(m, keys))
    table = torch.tensor([0, 1, 2, 9], dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="block_table entries"):
        codec.prepare_encode(k, v, toks, blobs, block_table=table, **_encode_kw(m, keys))
    # unchecked on the host: the device check fails the page at every call and writes its blob as zeros
    call = codec.prepare_encode(k, v, toks, blobs, block_table=table, check_block_table=False, **_encode_kw(m, keys))
    call()
    torch.cuda.synchronize()
    assert not blobs[3].any() and blobs[0].any()
    assert capi.PAGE_BAD_BLOCK == 6
