"""Session keyring (ztcp_b200.keyring) on CPU: the reference EphemeralSessionKeyRing's semantics with the
per-page tables in the C++ ledger.  Standalone checks of each rule, a differential run against the
reference class on random operation sequences (where the reference source is present), and the header
parser against struct.unpack."""
from __future__ import annotations

import os
import random
import struct
import sys

import numpy as np
import pytest

from ztcp_b200 import errors, ledger
from ztcp_b200.keyring import SessionKeyRing

PEPPER = b"p" * 32
REF_ROOT = os.environ.get("ZTCP_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                       "reference"))


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from ztcp_b200 import build

    build.build()


def egress(ring, t, s, model, layer, hg, base, toks):
    res, slots, last = ring.preflight_validate_egress(t, s, model, layer, hg, base, toks)
    try:
        ring.begin_egress_execution(t, s, res)
        ring.commit_egress(t, s, res, slots, last)
    finally:
        ring.release_egress_reservation(t, s, res)
    return last


def test_keys_and_nonce_ranges():
    ring = SessionKeyRing(PEPPER)
    enc, mac, k0, k1 = ring.derive_or_get("t", "s")
    assert len(enc) == 32 and len(mac) == 32 and (k0, k1) == struct.unpack("<QQ", bytes(enc[:16]))
    assert ring.derive_or_get("t", "s")[0] is enc
    assert ring.next_sequence_nonce("t", "s", 5) == 1
    assert ring.next_sequence_nonce("t", "s") == 6
    with pytest.raises(ValueError, match="count must be >= 1"):
        ring.next_sequence_nonce("t", "s", 0)
    with pytest.raises(ValueError, match="deployment_pepper"):
        SessionKeyRing(b"short")
    assert SessionKeyRing.pack_chacha20_nonce(2**64 + 7, 0x1234, 0xABCD) == struct.pack("<3I", 7, 0, 0x1234ABCD)


def test_nonce_reuse_and_stale_egress():
    ring = SessionKeyRing(PEPPER)
    toks = [11, 12, 13]
    assert egress(ring, "t", "s", 5, 3, 1, 100, toks) == 102
    with pytest.raises(errors.NonceReuseError, match="NONCE_REUSE_DETECTED"):
        ring.preflight_validate_egress("t", "s", 5, 3, 1, 102, [99])
    # slot (5, 3, 1, 12) is at version 101: an older version of it is stale
    with pytest.raises(errors.StalePageReplayError, match=r"stale sequence_nonce=50 < latest=101"):
        ring.preflight_validate_egress("t", "s", 5, 3, 1, 49, [77, 12])
    # a failed preflight burns nothing: the same range is still free for other slots
    egress(ring, "t", "s", 5, 3, 1, 49, [77, 78])
    # the same sequence nonces under another layer are different ChaCha20 nonces
    egress(ring, "t", "s", 5, 4, 1, 100, toks)
    with pytest.raises(ValueError, match="non-empty"):
        ring.preflight_validate_egress("t", "s", 5, 3, 1, 500, [])


def test_freshness_rules():
    ring = SessionKeyRing(PEPPER)
    egress(ring, "t", "s", 5, 3, 1, 10, [1, 2])
    gen, _, _ = ring.begin_ingress("t", "s")
    ring.verify_and_update_freshness("t", "s", 5, 3, 1, 1, 10, expected_generation=gen)  # re-read: fine
    ring.verify_and_update_freshness("t", "s", 5, 3, 1, 1, 20)                           # newer: raises mark
    with pytest.raises(errors.StalePageReplayError, match="is older than latest slot version=20"):
        ring.verify_and_update_freshness("t", "s", 5, 3, 1, 1, 10)
    with pytest.raises(errors.StalePageReplayError, match="!= expected_sequence_nonce=12"):
        ring.verify_and_update_freshness("t", "s", 5, 3, 1, 2, 11, expected_sequence_nonce=12)
    with pytest.raises(errors.StalePageReplayError, match="< min_sequence_nonce=30"):
        ring.verify_and_update_freshness("t", "s", 5, 3, 1, 2, 25, min_sequence_nonce=30)
    # batch: all or nothing
    with pytest.raises(errors.StalePageReplayError, match="older than latest slot version=20"):
        ring.verify_and_update_freshness_batch("t", "s", [(5, 3, 1, 2, 50), (5, 3, 1, 1, 19)])
    ring.verify_and_update_freshness("t", "s", 5, 3, 1, 2, 11)  # slot 2 was not raised to 50
    ring.verify_and_update_freshness_batch("t", "s", [(5, 3, 1, 2, 60), (5, 3, 1, 2, 60), (5, 3, 1, 1, 20)])
    with pytest.raises(errors.StalePageReplayError, match="< min_sequence_nonce=100"):
        ring.verify_and_update_freshness_batch("t", "s", [(5, 3, 1, 9, 99)], min_sequence_nonce=100)
    ring.finish_ingress("t", "s", gen)


def test_crypto_shred_revokes_and_resets():
    ring = SessionKeyRing(PEPPER)
    enc = ring.derive_or_get("t", "s")[0]
    ring.derive_or_get("t", "x")
    ring.derive_or_get("u", "s")
    res, slots, last = ring.preflight_validate_egress("t", "s", 1, 1, 1, 5, [1])
    gen, _, _ = ring.begin_ingress("t", "s")
    assert ring.crypto_shred_session("t", "s") is True
    assert not any(enc) and not any(res.enc_buf) and res.revoked
    with pytest.raises(errors.SessionShreddedError, match="before or during egress"):
        ring.begin_egress_execution("t", "s", res)
    with pytest.raises(errors.SessionShreddedError, match="before commit"):
        ring.commit_egress("t", "s", res, slots, last)
    ring.release_egress_reservation("t", "s", res)
    with pytest.raises(errors.SessionShreddedError, match="key is missing or crypto-shredded"):
        ring.begin_ingress("t", "s")
    with pytest.raises(errors.SessionShreddedError, match=f"generation {gen} was crypto-shredded during ingress"):
        ring.finish_ingress("t", "s", gen)
    assert ring.crypto_shred_session("t", "s") is False
    # a new generation starts with empty tables
    ring.derive_or_get("t", "s")
    assert ring.begin_ingress("t", "s")[0] == gen + 1
    assert ring.next_sequence_nonce("t", "s") == 1
    egress(ring, "t", "s", 1, 1, 1, 5, [1])
    assert ring.crypto_shred_tenant("t") == 2
    assert ring.crypto_shred_tenant("t") == 0


def test_custom_exception_classes():
    class Errs:
        class KVIntegrityError(RuntimeError): ...
        class CrossTenantContaminationError(KVIntegrityError): ...
        class StalePageReplayError(KVIntegrityError): ...
        class NonceReuseError(ValueError): ...
        class SessionShreddedError(RuntimeError): ...

    ring = SessionKeyRing(PEPPER, errors=Errs)
    egress(ring, "t", "s", 1, 1, 1, 5, [1])
    with pytest.raises(Errs.NonceReuseError):
        ring.preflight_validate_egress("t", "s", 1, 1, 1, 5, [2])
    with pytest.raises(Errs.SessionShreddedError):
        ring.begin_ingress("nobody", "s")


def test_header_records_match_struct():
    rng = np.random.default_rng(5)
    blobs = rng.integers(0, 256, (37, 70), dtype=np.uint8)
    rec = ledger.records_from_headers(blobs)
    for i in range(37):
        _, _, _, _, m, l_, g, tok, seq = struct.unpack_from("<HBBIIHHQQ", blobs[i].tobytes(), 0)
        assert (rec[i]["model_id_hash"], rec[i]["layer_id"], rec[i]["head_group_id"], rec[i]["page_token_hash"],
                rec[i]["sequence_nonce"]) == (m, l_, g, tok, seq)
    tup = ledger.records_from_tuples([(2**33 + 5, 2**17 + 3, 7, 2**64 + 9, 2**65 - 1)])
    assert tuple(tup[0]) == (5, 3, 7, 9, 2**64 - 1)


def test_batch_of_4096_pages_is_fast():
    import time

    ring = SessionKeyRing(PEPPER)
    toks = np.arange(1, 4097, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    t0 = time.perf_counter()
    res, slots, last = ring.preflight_validate_egress("t", "s", 1, 2, 3, 1000, toks)
    ring.commit_egress("t", "s", res, slots, last)
    ring.release_egress_reservation("t", "s", res)
    recs = np.zeros(4096, dtype=ledger.RECORD_DTYPE)
    recs["model_id_hash"], recs["layer_id"], recs["head_group_id"] = 1, 2, 3
    recs["page_token_hash"], recs["sequence_nonce"] = toks, 1000 + np.arange(4096, dtype=np.uint64)
    ring.verify_and_update_freshness_batch("t", "s", recs)
    assert time.perf_counter() - t0 < 0.5


# ---- differential run against the reference keyring ------------------------------------------------
@pytest.fixture(scope="module")
def ref_keyring():
    if not os.path.isdir(os.path.join(REF_ROOT, "research", "baseline_codec")):
        pytest.skip("reference source not present")
    sys.path.insert(0, REF_ROOT)
    from research.baseline_codec import fused_quant_crypto

    return fused_quant_crypto


def _outcome(fn):
    try:
        r = fn()
    except Exception as e:  # noqa: BLE001
        return ("raise", type(e).__name__, str(e))
    return ("ok", r)


@pytest.mark.parametrize("seed", range(int(os.environ.get("ZTCP_KEYRING_SEEDS", "12"))))
def test_matches_reference_keyring(ref_keyring, seed):
    rng = random.Random(seed)
    ref = ref_keyring.EphemeralSessionKeyRing(deployment_pepper=PEPPER)
    ours = SessionKeyRing(PEPPER, errors=ref_keyring)
    sessions = [("ta", "s1"), ("ta", "s2"), ("tb", "s1")]
    pending = {id(ref): [], id(ours): []}
    gens = {}
    for step in range(150):
        t, s = rng.choice(sessions)
        op = rng.choice(["next", "egress", "egress", "egress", "stage", "finish_staged", "fresh", "fresh_batch",
                         "shred", "shred_tenant", "ingress"])
        model, layer, hg = rng.choice([1, 2]), rng.choice([0, 7]), rng.choice([0, 3])
        toks = [rng.choice([10, 11, 12, 13, 2**64 - 1]) for _ in range(rng.randint(1, 4))]
        base = rng.choice([1, 2, 5, 8, 20, 40, 2**64 - 2])
        rng_count = rng.randint(1, 3)
        rng_seq = rng.choice([1, 3, 6, 10, 25, 60])
        rng_min = rng.choice([None, None, 4, 30])
        rng_exp = rng.choice([None, None, None, rng_seq])
        outs = []
        for ring in (ref, ours):
            if op == "next":
                outs.append(_outcome(lambda: ring.next_sequence_nonce(t, s, rng_count)))
            elif op == "egress":
                outs.append(_outcome(lambda: egress(ring, t, s, model, layer, hg, base, toks)))
            elif op == "stage":
                o = _outcome(lambda: ring.preflight_validate_egress(t, s, model, layer, hg, base, toks))
                if o[0] == "ok":
                    pending[id(ring)].append((t, s, o[1]))
                    o = ("ok", o[1][2])
                outs.append(o)
            elif op == "finish_staged":
                if pending[id(ring)]:
                    pt, ps, (res, slots, last) = pending[id(ring)].pop(0)

                    def fin():
                        try:
                            ring.begin_egress_execution(pt, ps, res)
                            ring.commit_egress(pt, ps, res, slots, last)
                        finally:
                            ring.release_egress_reservation(pt, ps, res)
                        return last
                    outs.append(_outcome(fin))
                else:
                    outs.append(("none",))
            elif op == "fresh":
                seq = rng_seq
                outs.append(_outcome(lambda: ring.verify_and_update_freshness(
                    t, s, model, layer, hg, toks[0], seq, min_sequence_nonce=rng_min, expected_sequence_nonce=rng_exp,
                    expected_generation=gens.get((id(ring), t, s)))))
            elif op == "fresh_batch":
                recs = [(model, layer, hg, tk, rng_seq + j) for j, tk in enumerate(toks)]
                outs.append(_outcome(lambda: ring.verify_and_update_freshness_batch(
                    t, s, recs, min_sequence_nonce=rng_min, expected_generation=gens.get((id(ring), t, s)))))
            elif op == "shred":
                outs.append(_outcome(lambda: ring.crypto_shred_session(t, s)))
            elif op == "shred_tenant":
                outs.append(_outcome(lambda: ring.crypto_shred_tenant(t)))
            elif op == "ingress":
                o = _outcome(lambda: ring.begin_ingress(t, s))
                if o[0] == "ok":
                    gens[(id(ring), t, s)] = o[1][0]
                    o = ("ok", o[1][0], len(o[1][1]), len(o[1][2]))
                outs.append(o)
        assert outs[0] == outs[1], (seed, step, op, outs)
