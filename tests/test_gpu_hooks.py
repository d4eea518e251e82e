"""Per-page fallback decode (the C-ABI's ZTCP_OPT_PAGE_FALLBACK) and the offload hooks over it: a tampered,
cross-tenant or malformed page is zeroed and reported while the other pages of the batch decode to the
oracle's output; stale replays and shredded sessions become misses in the hook's hit bitmap."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _encode(oracle, n, seed):
    from ztcp_b200 import workload

    m = workload.session_material(seed)
    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=seed)
    k16, v16 = k32.astype(np.float16), v32.astype(np.float16)
    toks = workload.token_hashes(n, seed + 1)
    want = helpers.oracle_encode(oracle, k16, v16, toks, 64, 1, 1, 98304, m)
    return m, k16, v16, toks, want


def test_page_fallback_decodes_the_passing_pages(oracle):
    from ztcp_b200 import build, capi, codec

    build.build()

    n = 6
    m, k16, v16, toks, want = _encode(oracle, n, 41)
    bad = want.copy()
    bad[1, 5000] ^= 0x01            # ciphertext bit flip -> MAC failure
    bad[3, 4] ^= 0x01               # tenant hash in the header -> AAD mismatch
    bad[4, 3] = 0x44                # flags byte changed without a new tag: the MAC check (before flags) fails
    okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k16.shape, 64, False, m)
    assert first == -1
    keys = capi.keys(*m["key"], *m["mac_key"])
    for fallback in (True, False):
        ko = torch.full(k16.shape, 7.0, dtype=torch.float16, device=DEV)
        vo = torch.full(k16.shape, 7.0, dtype=torch.float16, device=DEV)
        status, fail = codec.decode_pages(torch.from_numpy(bad).to(DEV), torch.from_numpy(toks.view(np.int64)).to(DEV),
                                          ko, vo, rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"],
                                          model_id_hash=m["model"], layer_id=m["layer"], keys=keys,
                                          page_fallback=fallback)
        st = status.cpu().numpy()
        assert list(st) == [0, capi.PAGE_MAC_FAILED, 0, capi.PAGE_AAD_MISMATCH, capi.PAGE_MAC_FAILED, 0]
        assert int(fail.item()) == 1
        kh, vh = ko.cpu().numpy().view(np.uint16), vo.cpu().numpy().view(np.uint16)
        for i in range(n):
            if fallback and st[i] == 0:
                np.testing.assert_array_equal(kh[i], okd[i])
                np.testing.assert_array_equal(vh[i], ovd[i])
            else:
                assert not kh[i].any() and not vh[i].any()


@pytest.fixture()
def hook():
    from ztcp_b200 import build
    from ztcp_b200.cold_page_spec import ColdPageGeometry
    from ztcp_b200.hooks import CompactStagingRing, HiCachePageCodec
    from ztcp_b200.keyring import SessionKeyRing
    from ztcp_b200.session import ColdPageCodec

    build.build()
    geom = ColdPageGeometry(num_tokens=64, num_kv_heads=8, head_dim=128, rope_dim=64)
    ring = SessionKeyRing(b"h" * 32)
    sc = ColdPageCodec(geom, ring, DEV)
    return HiCachePageCodec(sc, CompactStagingRing(32, 98352)), ring


def _aad(seq):
    from ztcp_b200.cold_page_spec import ColdPageAAD, QuantPreset, RoPEMode, hash32

    return ColdPageAAD(hash32("tenant-h"), hash32("model-h"), 9, 0, seq, QuantPreset.INT4_SYM, RoPEMode.PRESERVE_FP8, 2)


def test_hook_store_load_and_per_page_misses(hook):
    from ztcp_b200 import workload

    hc, ring = hook
    n = 8
    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=77)
    k, v = torch.from_numpy(k32).to(torch.bfloat16).to(DEV), torch.from_numpy(v32).to(torch.bfloat16).to(DEV)
    toks = torch.from_numpy(workload.token_hashes(n, 78).view(np.int64)).to(DEV)
    seq = ring.next_sequence_nonce("tenant-h", "s", n)
    view = hc.store(k, v, toks, "tenant-h", "s", _aad(seq))
    view.ready.synchronize()
    # the same blobs through the all-or-nothing decoder: the reference result for every page
    ref_k, ref_v = hc.codec.decode_cold_pages_batch_tensor(view.blobs.clone().to(DEV), toks, "tenant-h", "s",
                                                           "model-h", 9)
    view.blobs[2, 6000] ^= 0x80  # tamper one staged page
    ko = torch.full(tuple(k.shape), 3.0, dtype=torch.float16, device=DEV)
    vo = torch.full(tuple(k.shape), 3.0, dtype=torch.float16, device=DEV)
    hits = hc.load(view, ko, vo, "tenant-h", "s", "model-h", 9)
    assert hits.dtype == torch.bool and hits.tolist() == [i != 2 for i in range(n)]
    assert not ko[2].any() and not vo[2].any()
    keep = torch.tensor([i for i in range(n) if i != 2], device=DEV)
    assert torch.equal(ko[keep], ref_k[keep]) and torch.equal(vo[keep], ref_v[keep])

    # a newer version of the same page slots: loading it advances the watermarks, the old view is stale
    seq2 = ring.next_sequence_nonce("tenant-h", "s", n)
    view2 = hc.store(k, v, toks, "tenant-h", "s", _aad(seq2))
    hits2 = hc.load(view2, ko, vo, "tenant-h", "s", "model-h", 9)
    assert hits2.all()
    view.blobs[2, 6000] ^= 0x80  # untampered again, but older than the slot watermarks now
    hits_old = hc.load(view, ko, vo, "tenant-h", "s", "model-h", 9)
    assert not hits_old.any() and not ko.any() and not vo.any()

    # a shredded session: every page is a miss
    ring.crypto_shred_session("tenant-h", "s")
    ko.fill_(1.0)
    assert not hc.load(view2, ko, vo, "tenant-h", "s", "model-h", 9).any()
    assert not ko.any()
    hc.ring.release(view)
    hc.ring.release(view2)
    assert hc.ring.free_slots == 32


def test_page_fallback_random_sweep(oracle):
    """Per-page fallback decode on 30 seeded random configurations with random pages tampered (ciphertext
    bit, tenant byte of the header, magic): statuses equal the oracle's, every untampered page equals the
    oracle's decode of the untouched blobs, every tampered page is zero, and the batch flag is set."""
    from ztcp_b200 import build, capi, codec, workload

    build.build()
    rng = np.random.default_rng(777)
    for case in range(30):
        D = int(rng.choice([16, 48, 64, 128, 576]))
        T, H = int(rng.integers(1, 33)), int(rng.integers(1, 9 if D <= 128 else 2))
        rope = int(rng.integers(0, D // 16 + 1)) * 16
        rope_mode = int(rng.integers(0, 3)) if rope > 0 else 0
        preset, mla, n = int(rng.integers(1, 4)), bool(rng.random() < 0.3), int(rng.integers(2, 7))
        k16 = rng.standard_normal((n, T, H, D)).astype(np.float16)
        v16 = None if mla else rng.standard_normal((n, T, H, D)).astype(np.float16)
        m = workload.session_material(int(rng.integers(1 << 30)))
        toks = workload.token_hashes(n, int(rng.integers(1 << 30)))
        exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla)
        clean = helpers.oracle_encode(oracle, k16, v16, toks, rope, preset, rope_mode, exp, m)
        okd, ovd, _, first = helpers.oracle_decode(oracle, clean, toks, k16.shape, rope, mla, m)
        assert first == -1
        bad = clean.copy()
        tampered = rng.choice(n, int(rng.integers(1, n)), replace=False)
        for i in tampered:
            kind = int(rng.integers(0, 3))
            if kind == 0:
                bad[i, 32 + int(rng.integers(0, exp))] ^= 1 << int(rng.integers(0, 8))  # ciphertext
            elif kind == 1:
                bad[i, 4] ^= 0x01  # tenant hash
            else:
                bad[i, 0] ^= 0x01  # magic
        _, _, ost, _ = helpers.oracle_decode(oracle, bad, toks, k16.shape, rope, mla, m)
        ko = torch.full(k16.shape, 3.0, dtype=torch.float16, device=DEV)
        vo = None if mla else torch.full(k16.shape, 3.0, dtype=torch.float16, device=DEV)
        status, fail = codec.decode_pages(torch.from_numpy(bad).to(DEV), torch.from_numpy(toks.view(np.int64)).to(DEV),
                                          ko, vo, rope_dim=rope, is_mla=mla, tenant_id_hash=m["tenant"],
                                          model_id_hash=m["model"], layer_id=m["layer"],
                                          keys=capi.keys(*m["key"], *m["mac_key"]), page_fallback=True)
        tag = f"case {case}: T{T} H{H} D{D} rope{rope} preset{preset} mode{rope_mode} mla{mla} n{n} bad{sorted(tampered)}"
        st = status.cpu().numpy()
        np.testing.assert_array_equal(st, np.asarray(ost), err_msg=tag)
        assert int(fail.item()) == 1, tag
        kh = ko.cpu().numpy().view(np.uint16)
        vh = None if mla else vo.cpu().numpy().view(np.uint16)
        for i in range(n):
            if st[i] == 0:
                np.testing.assert_array_equal(kh[i], okd[i], err_msg=tag)
                if not mla:
                    np.testing.assert_array_equal(vh[i], ovd[i], err_msg=tag)
            else:
                assert not kh[i].any() and (mla or not vh[i].any()), tag
