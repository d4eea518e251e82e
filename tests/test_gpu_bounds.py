"""Device-side checks and measurement entry points through the C-ABI.

* A block-table entry outside [0, kv_pool_pages) is caught by the kernels before any access: encode
  writes that page's blob as zeros, decode reports ZTCP_PAGE_BAD_BLOCK and never touches memory outside
  the pool.  The pool sits between two guard pages of the same allocation, so an unchecked entry of -1 or
  pool_pages would land in a guard (never outside the test's own memory) and show up as a changed guard.
* ztcp_measure_int_peaks measures the integer ceilings of the codec's primitives; ztcp_mark_phase splits a
  codec call's time between its two kernels."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_block_table_entries_outside_the_pool_are_rejected_on_the_device(oracle):
    from ztcp_b200 import capi, codec, workload

    pool = 6
    k32, v32 = workload.kv_pages_np(pool + 2, workload.GQA, seed=51)
    kbuf = torch.from_numpy(k32).to(torch.bfloat16).to(DEV)   # [guard, pool pages..., guard]
    vbuf = torch.from_numpy(v32).to(torch.bfloat16).to(DEV)
    kpool, vpool = kbuf[1:pool + 1], vbuf[1:pool + 1]
    table = torch.tensor([0, pool, 2, -1, 5], dtype=torch.int32, device=DEV)
    n = table.numel()
    m = workload.session_material(52)
    toks = workload.token_hashes(n, 53)
    keys = capi.keys(*m["key"], *m["mac_key"])
    td = torch.from_numpy(toks).to(DEV)
    blobs = torch.full((n, 98352), 0xA5, dtype=torch.uint8, device=DEV)
    codec.encode_pages(kpool, vpool, td, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                       head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys, block_table=table,
                       check_block_table=False)
    got = blobs.cpu().numpy()
    k16, v16 = kpool.half().cpu().numpy(), vpool.half().cpu().numpy()
    for i, blk in enumerate(table.tolist()):
        if 0 <= blk < pool:
            want = helpers.oracle_encode(oracle, k16[blk][None], v16[blk][None], toks[i:i + 1], 64, 1, 1, 98304,
                                         dict(m, base_seq=(m["base_seq"] + i) % 2**64))
            np.testing.assert_array_equal(got[i], want[0], err_msg=f"page {i}")
        else:
            assert not got[i].any(), f"page {i} (block {blk}) must be written as zeros"

    guard = 0x3C00  # fp16 1.0 in every element of both guard pages
    for fallback in (False, True):
        obuf_k = torch.full((pool + 2, 64, 8, 128), 2.0, dtype=torch.float16, device=DEV)
        obuf_v = torch.full_like(obuf_k, 2.0)
        for ob in (obuf_k, obuf_v):
            ob[0].fill_(1.0)
            ob[pool + 1].fill_(1.0)
        st, fail = codec.decode_pages(blobs, td, obuf_k[1:pool + 1], obuf_v[1:pool + 1], rope_dim=64, is_mla=False,
                                      tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                                      keys=keys, block_table=table, check_block_table=False, page_fallback=fallback)
        torch.cuda.synchronize()
        assert st.cpu().tolist() == [0, capi.PAGE_BAD_BLOCK, 0, capi.PAGE_BAD_BLOCK, 0]
        assert int(fail.item()) == 1
        for ob in (obuf_k, obuf_v):
            for gp in (0, pool + 1):
                assert (ob[gp].view(torch.int16) == guard).all(), "a guard page outside the pool was written"
        for i, blk in enumerate(table.tolist()):
            if not 0 <= blk < pool:
                continue
            kd, vd = obuf_k[1 + blk], obuf_v[1 + blk]
            if fallback:
                okd, ovd, _, first = helpers.oracle_decode(oracle, got[i:i + 1], toks[i:i + 1], (1, 64, 8, 128), 64,
                                                           False, m)
                assert first == -1
                np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd[0])
                np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd[0])
            else:
                assert not kd.any() and not vd.any(), "a failed batch zeroes every in-pool output page"
        with pytest.raises(RuntimeError, match="outside the KV pool"):
            codec.raise_for_status(st, fail)


def test_int_peaks_are_measured():
    from ztcp_b200 import capi

    lib = capi.load()
    scratch = torch.empty(capi.MEASURE_SCRATCH_BYTES, dtype=torch.uint8, device=DEV)
    p = capi.IntPeaks()
    capi.check(lib.ztcp_measure_int_peaks(scratch.data_ptr(), scratch.numel(), C.byref(p)))
    assert p.sms == torch.cuda.get_device_properties(0).multi_processor_count
    # ranges around the figures measured on B200 (2.9e10 blocks/s, 4.2e11 words/s, 89 cycles/word)
    assert 5e9 < p.chacha20_blocks_per_s < 1e11
    assert 1e11 < p.sip_words_per_s < 2e12
    assert 40 < p.sip_chain_cycles_per_word < 400
    assert 0.1 < p.sip_chain_ms < 5


def test_phase_mark_splits_a_call_between_its_kernels():
    from ztcp_b200 import capi, codec, workload

    lib = capi.load()
    n = 16
    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=61)
    kb = torch.from_numpy(k32).to(torch.bfloat16).to(DEV)
    vb = torch.from_numpy(v32).to(torch.bfloat16).to(DEV)
    m = workload.session_material(62)
    keys = capi.keys(*m["key"], *m["mac_key"])
    td = torch.from_numpy(workload.token_hashes(n, 63)).to(DEV)
    blobs = torch.empty((n, 98352), dtype=torch.uint8, device=DEV)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    ev[0].record()
    capi.check(lib.ztcp_mark_phase(C.c_void_p(ev[1].cuda_event)))
    codec.encode_pages(kb, vb, td, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                       head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
    ev[2].record()
    torch.cuda.synchronize()
    tile, chain = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    assert 0 < tile < chain, (tile, chain)   # the tag chain (~0.6 ms) outlasts a 16-page tile kernel
    assert chain > 0.2
    # the mark is one-shot: a second call records nothing on the event
    stamp = torch.cuda.Event(enable_timing=True)
    stamp.record()
    torch.cuda.synchronize()
    codec.encode_pages(kb, vb, td, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                       head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
    torch.cuda.synchronize()
    assert stamp.elapsed_time(ev[1]) < 0
