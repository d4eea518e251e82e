"""GPU-native session codec (ztcp_b200.session.ColdPageCodec) with the C++-ledger keyring: the reference
wrapper's interface on CUDA tensors.  Wire bytes equal the oracle's under the session's derived keys; the
keyring protocol's failures surface as the reference's exceptions with outputs zeroed."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def parts():
    from ztcp_b200 import build, workload
    from ztcp_b200.cold_page_spec import ColdPageAAD, ColdPageGeometry, QuantPreset, RoPEMode, hash32
    from ztcp_b200.keyring import SessionKeyRing
    from ztcp_b200.session import ColdPageCodec

    build.build()
    geom = ColdPageGeometry(num_tokens=64, num_kv_heads=8, head_dim=128, rope_dim=64)
    ring = SessionKeyRing(b"z" * 32)
    return dict(workload=workload, AAD=ColdPageAAD, geom=geom, ring=ring, codec=ColdPageCodec(geom, ring, DEV),
                P=QuantPreset, R=RoPEMode, hash32=hash32)


def _aad(p, seq, layer=5, token=0):
    return p["AAD"](p["hash32"]("tenant-a"), p["hash32"]("model-x"), layer, token, seq, p["P"].INT4_SYM,
                    p["R"].PRESERVE_FP8, 3)


def _material(p, tenant, session, aad):
    enc, mac, _, _ = p["ring"].derive_or_get(tenant, session)
    return {"key": list(struct.unpack("<QQQQ", bytes(enc))), "mac_key": list(struct.unpack("<QQ", bytes(mac[:16]))),
            "tenant": aad.tenant_id_hash, "model": aad.model_id_hash, "layer": aad.layer_id,
            "head_group": aad.head_group_id, "base_seq": aad.sequence_nonce}


def test_batch_round_trip_matches_oracle(parts, oracle):
    p = parts
    k32, v32 = p["workload"].kv_pages_np(16, p["workload"].GQA, seed=3)
    kb = torch.from_numpy(k32).to(torch.bfloat16)
    vb = torch.from_numpy(v32).to(torch.bfloat16)
    toks = torch.from_numpy(p["workload"].token_hashes(16, 9).view(np.int64))
    seq = p["ring"].next_sequence_nonce("tenant-a", "s1", 16)
    aad = _aad(p, seq)
    blobs = p["codec"].encode_cold_pages_batch_tensor(kb.to(DEV), vb.to(DEV), toks.to(DEV), "tenant-a", "s1", aad)
    torch.cuda.synchronize()
    want = helpers.oracle_encode(oracle, kb.half().numpy(), vb.half().numpy(), toks.numpy().view(np.uint64), 64, 1, 1,
                                 98304, _material(p, "tenant-a", "s1", aad))
    np.testing.assert_array_equal(blobs.cpu().numpy(), want)
    k_out = torch.full(tuple(kb.shape), 7.0, dtype=torch.float16, device=DEV)
    v_out = torch.full(tuple(kb.shape), 7.0, dtype=torch.float16, device=DEV)
    p["codec"].decode_cold_pages_peak_into(blobs, toks.to(DEV), k_out, v_out, "tenant-a", "s1", "model-x", 5)
    okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks.numpy().view(np.uint64), tuple(kb.shape), 64, False,
                                               _material(p, "tenant-a", "s1", aad))
    assert first == -1
    np.testing.assert_array_equal(k_out.cpu().numpy().view(np.uint16), okd)
    np.testing.assert_array_equal(v_out.cpu().numpy().view(np.uint16), ovd)
    # CPU tensors through the same codec: staged to the GPU, results back on the CPU
    k2, v2 = p["codec"].decode_cold_pages_batch_tensor(blobs.cpu(), toks, "tenant-a", "s1", "model-x", 5)
    assert k2.device.type == "cpu" and torch.equal(k2, k_out.cpu()) and torch.equal(v2, v_out.cpu())


def test_failures_raise_reference_errors_and_zero(parts):
    from ztcp_b200 import errors

    p = parts
    k32, v32 = p["workload"].kv_pages_np(4, p["workload"].GQA, seed=5)
    k = torch.from_numpy(k32).half().to(DEV)
    v = torch.from_numpy(v32).half().to(DEV)
    toks = torch.from_numpy(p["workload"].token_hashes(4, 21).view(np.int64)).to(DEV)
    base = p["ring"].next_sequence_nonce("tenant-a", "s2", 8)
    old = p["codec"].encode_cold_pages_batch_tensor(k, v, toks, "tenant-a", "s2", _aad(p, base))
    new = p["codec"].encode_cold_pages_batch_tensor(k, v, toks, "tenant-a", "s2", _aad(p, base + 4))
    # an older version of the same slots is refused before its nonces are checked ...
    with pytest.raises(errors.StalePageReplayError, match="Cannot encode cold page with stale"):
        p["codec"].encode_cold_pages_batch_tensor(k, v, toks, "tenant-a", "s2", _aad(p, base))
    # ... and fresh slots cannot reuse burned nonces
    toks2 = torch.from_numpy(p["workload"].token_hashes(4, 22).view(np.int64)).to(DEV)
    with pytest.raises(errors.NonceReuseError, match="NONCE_REUSE_DETECTED"):
        p["codec"].encode_cold_pages_batch_tensor(k, v, toks2, "tenant-a", "s2", _aad(p, base))
    ko = torch.ones((4, 64, 8, 128), dtype=torch.float16, device=DEV)
    vo = torch.ones_like(ko)
    p["codec"].decode_cold_pages_peak_into(new, toks, ko, vo, "tenant-a", "s2", "model-x", 5)
    # the superseded version of the same slots is a stale replay: outputs zeroed
    with pytest.raises(errors.StalePageReplayError, match="older than latest slot version"):
        p["codec"].decode_cold_pages_peak_into(old, toks, ko, vo, "tenant-a", "s2", "model-x", 5)
    assert not ko.any() and not vo.any()
    bad = new.clone()
    bad[2, 500] ^= 1
    with pytest.raises(errors.KVIntegrityError, match="MAC verification failed"):
        p["codec"].decode_cold_pages_peak_into(bad, toks, ko, vo, "tenant-a", "s2", "model-x", 5)
    with pytest.raises(errors.CrossTenantContaminationError, match="AAD mismatch"):
        p["codec"].decode_cold_pages_peak_into(new, toks, ko, vo, "tenant-a", "s2", "model-y", 5)
    # single page: expected-nonce check, then crypto-shred
    one = p["codec"].encode_cold_page_tensor(k[0], v[0], "tenant-a", "s2", _aad(p, base + 100, token=77))
    kk, vv = p["codec"].decode_cold_page_tensor(one, "tenant-a", "s2", "model-x", 5, 77,
                                                expected_sequence_nonce=base + 100)
    assert kk.shape == (64, 8, 128) and kk.any()
    with pytest.raises(errors.StalePageReplayError, match="!= expected_sequence_nonce"):
        p["codec"].decode_cold_page_tensor(one, "tenant-a", "s2", "model-x", 5, 77, expected_sequence_nonce=base)
    p["ring"].crypto_shred_session("tenant-a", "s2")
    with pytest.raises(errors.SessionShreddedError):
        p["codec"].decode_cold_pages_peak_into(new, toks, ko, vo, "tenant-a", "s2", "model-x", 5)
