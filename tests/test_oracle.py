"""Pin the CPU oracle: golden vectors from the reference, and the reference build itself."""
from __future__ import annotations

import itertools
import struct

import numpy as np
import pytest

import helpers


def test_chacha20_kats(oracle):
    for v in helpers.load_json("kat_chacha20.json"):
        out = oracle.chacha20_xor(bytes.fromhex(v["data"]), bytes.fromhex(v["key"]), v["counter"],
                                  bytes.fromhex(v["nonce"]))
        assert out.hex() == v["out"]


def test_siphash_kats(oracle):
    for v in helpers.load_json("kat_siphash.json"):
        k0, k1 = struct.unpack("<QQ", bytes.fromhex(v["key"]))
        assert oracle.siphash24_128(bytes.fromhex(v["data"]), k0, k1).hex() == v["tag"]


def test_codec_small_golden(oracle):
    cases, arrays = helpers.small_cases()
    assert len(cases) >= 100
    for c in cases:
        i = c["id"]
        k = arrays[f"k{i}"].reshape(-1, c["T"], c["H"], c["D"])
        v = None if c["mla"] else arrays[f"v{i}"].reshape(k.shape)
        toks = arrays[f"tok{i}"]
        blobs = helpers.oracle_encode(oracle, k, v, toks, c["rope"], c["preset"], c["rope_mode"],
                                      c["expected_payload"], c["material"])
        np.testing.assert_array_equal(blobs, arrays[f"blobs{i}"], err_msg=f"encode case {c}")
        kd, vd, st, first = helpers.oracle_decode(oracle, arrays[f"blobs{i}"], toks, k.shape, c["rope"], c["mla"],
                                                  c["material"])
        assert first == -1 and not st.any()
        np.testing.assert_array_equal(kd, arrays[f"kdec{i}"].reshape(kd.shape), err_msg=f"decode case {c}")
        if not c["mla"]:
            np.testing.assert_array_equal(vd, arrays[f"vdec{i}"].reshape(vd.shape))


@pytest.mark.parametrize("case", helpers.load_json("codec_digests.json"), ids=lambda c: c["name"])
def test_full_size_digests(oracle, case):
    kb, vb, k16, v16, m, toks, shape = helpers.full_case_inputs(case)
    assert helpers.sha(kb.view(__import__("torch").int16).numpy()) == case["input_bf16_sha256"][:64]
    blobs = helpers.oracle_encode(oracle, k16.numpy(), None if v16 is None else v16.numpy(), toks, shape.rope_dim,
                                  case["preset"], case["rope_mode"], case["expected_payload"], m)
    assert blobs.shape[1] == case["blob_bytes"]
    assert helpers.sha(blobs) == case["blobs_sha256"]
    kd, vd, st, first = helpers.oracle_decode(oracle, blobs, toks, tuple(k16.shape), shape.rope_dim, shape.mla, m)
    assert first == -1
    assert helpers.sha(kd) == case["k_decoded_sha256"]
    if vd is not None:
        assert helpers.sha(vd) == case["v_decoded_sha256"]


def test_blob_sizes_match_published(oracle):
    # latest_results.json:114-116 / RESULTS_LOG.md:42-44: GQA INT4+FP8 98,352 B, K8V4+FP8 114,736 B
    assert 48 + oracle.spec_payload_bytes(1, 1, 512, 128, 64, True) == 98352
    assert 48 + oracle.spec_payload_bytes(2, 1, 512, 128, 64, True) == 114736
    assert 48 + oracle.spec_payload_bytes(1, 1, 64, 576, 64, False) == 25136


def test_decode_status_order(oracle):
    """magic -> AAD -> MAC -> flags -> length, as the reference's batch decoder checks (csrc:2309-2355)."""
    from ztcp_b200 import workload

    m = workload.session_material(3)
    rng = np.random.default_rng(5)
    k = rng.standard_normal((3, 2, 2, 32)).astype(np.float16)
    v = rng.standard_normal((3, 2, 2, 32)).astype(np.float16)
    toks = workload.token_hashes(3, 9)
    exp = oracle.spec_payload_bytes(1, 1, 4, 32, 16, True)
    blobs = helpers.oracle_encode(oracle, k, v, toks, 16, 1, 1, exp, m)

    def dec(b, t=toks, **over):
        mm = dict(m, **over)
        return helpers.oracle_decode(oracle, b, t, k.shape, 16, False, mm)

    _, _, st, first = dec(blobs)
    assert first == -1
    bad = blobs.copy(); bad[1, 0] ^= 1
    assert dec(bad)[2].tolist() == [0, 1, 0]
    bad = blobs.copy(); bad[2, 40] ^= 0x80
    kd, vd, st, first = dec(bad)
    assert st.tolist() == [0, 0, 3] and first == 2 and not kd.any() and not vd.any()
    assert dec(blobs, layer=m["layer"] ^ 1)[2].tolist() == [2, 2, 2]
    t2 = toks.copy(); t2[0] ^= 1
    assert dec(blobs, t=t2)[2].tolist() == [2, 0, 0]
    # valid tag over an invalid flags byte -> 4; a payload shorter than the flags need -> 5
    forged = blobs.copy(); forged[0, 3] = 0x05
    forged[0, -16:] = np.frombuffer(oracle.siphash24_128(forged[0, :-16].tobytes(), *m["mac_key"]), np.uint8)
    assert dec(forged)[2].tolist() == [4, 0, 0]
    short = np.concatenate([blobs[:, :32 + 40], blobs[:, -16:]], axis=1)
    for b in range(3):
        short[b, -16:] = np.frombuffer(oracle.siphash24_128(short[b, :-16].tobytes(), *m["mac_key"]), np.uint8)
    assert dec(short)[2].tolist() == [5, 5, 5]


def test_scale_division_forms_agree():
    """fp16(amax / d) == fp16(amax * (1/d)) for every non-negative finite fp16 amax, the 1e-6 floor and inf,
    d in {7, 127}: the reference's -ffast-math build may use either form."""
    h = np.arange(0, 0x7C01, dtype=np.uint16).view(np.float16).astype(np.float32)
    vals = np.concatenate([h, np.array([1e-6], np.float32)])
    for d in (np.float32(7.0), np.float32(127.0)):
        a = (vals / d).astype(np.float16)
        b = (vals * (np.float32(1.0) / d)).astype(np.float16)
        assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def _ref_module():
    import build_ref

    try:
        return build_ref.load_module()
    except FileNotFoundError:
        return None


@pytest.mark.parametrize("preset,rope_mode,mla", list(itertools.product([1, 2, 3], [0, 1, 2], [False, True])))
def test_oracle_matches_reference_build(oracle, preset, rope_mode, mla):
    """Randomized differential test against the reference codec compiled from its own source."""
    ref = _ref_module()
    if ref is None:
        pytest.skip("oracle/_ref not built (run python oracle/build_ref.py where the reference is present)")
    import torch

    from ztcp_b200 import workload

    rng = np.random.default_rng(preset * 100 + rope_mode * 10 + mla)
    for T, H, D, rope in [(4, 2, 64, 16), (3, 3, 128, 64), (2, 1, 80, 32)]:
        k = (rng.standard_normal((3, T, H, D)) * rng.choice([1e-3, 1.0, 100.0])).astype(np.float16)
        k[0, 0, 0, :16] = 0
        v = None if mla else rng.standard_normal((3, T, H, D)).astype(np.float16)
        m = workload.session_material(int(rng.integers(1 << 30)))
        toks = workload.token_hashes(3, int(rng.integers(1 << 30)))
        exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla) + int(rng.integers(0, 3)) * 4
        out = torch.zeros((3, 48 + exp), dtype=torch.uint8)
        ref.fused_encode_cold_pages_peak_into_cpu(
            torch.from_numpy(k), None if v is None else torch.from_numpy(v), torch.from_numpy(toks), out, preset,
            rope_mode, rope, exp, m["tenant"], m["model"], m["layer"], m["head_group"], m["base_seq"], m["key"][0],
            m["key"][1], m["mac_key"][0], m["mac_key"][1], m["key"][2], m["key"][3])
        mine = helpers.oracle_encode(oracle, k, v, toks, rope, preset, rope_mode, exp, m)
        np.testing.assert_array_equal(mine, out.numpy())


def _neon_group(x16: np.ndarray, qmax: int):
    """Independent numpy restatement of the reference's ARM NEON group quantizer (fp16 arithmetic)."""
    a = np.abs(x16.astype(np.float32))
    m = a[0]
    for val in a[1:]:
        m = np.float32(np.nan) if (np.isnan(m) or np.isnan(val)) else max(m, val)
    amax = np.float32(1e-6) if m < np.float32(1e-6) else m
    sh = np.float16(np.float32(amax) * (np.float32(1.0) / np.float32(qmax)))
    with np.errstate(all="ignore"):
        inv = np.float16(np.float32(1.0) / np.float32(sh))
        p = (x16.astype(np.float32) * np.float32(inv)).astype(np.float16).astype(np.float32)
    s = np.where(np.isnan(p), 0, np.clip(np.rint(np.nan_to_num(p, nan=0.0)), -32768, 32767)).astype(np.int32)
    if qmax == 127:
        q = np.maximum(np.clip(s, -128, 127), -127).astype(np.int8).view(np.uint8)
        return q, sh
    u = np.minimum(np.clip((s + 8).astype(np.int16).astype(np.int32), 0, 255), 15)
    return (u[0::2] | (u[1::2] << 4)).astype(np.uint8), sh


@pytest.mark.parametrize("preset", [1, 3])
def test_neon_mode_matches_numpy_restatement(oracle, preset):
    from ztcp_b200 import workload

    rng = np.random.default_rng(preset)
    edge = np.array([np.inf, -np.inf, np.nan, 65504, -65504, 7e4, 1e-7, -6e-8, 0.0, 3.0e-5], dtype=np.float32)
    m = workload.session_material(9)
    qmax = 7 if preset == 1 else 127
    qb = 8 if preset == 1 else 16
    for trial in range(300):
        scale_mag = 10.0 ** rng.uniform(-9, 5)
        x = (rng.standard_normal((2, 16)) * scale_mag).astype(np.float32)
        if trial % 3 == 0:
            x.flat[rng.integers(0, 32, 3)] = rng.choice(edge, 3)
        with np.errstate(over="ignore"):  # magnitudes beyond 65504 become inf on purpose
            x16 = x.astype(np.float16)
        k = x16[0].reshape(1, 1, 1, 16)
        v = x16[1].reshape(1, 1, 1, 16)
        exp = oracle.spec_payload_bytes(preset, 0, 1, 16, 0, True)
        blob = oracle.encode_batch(k.view(np.uint16), v.view(np.uint16), np.array([5], np.uint64), rope_dim=0,
                                   preset=preset, rope_mode=0, expected_payload=exp, tenant=1, model=2, layer=3,
                                   head_group=4, base_seq=trial, key=m["key"], mac_key=m["mac_key"], neon=True)[0]
        key32 = b"".join(int(w).to_bytes(8, "little") for w in m["key"])
        nonce = struct.pack("<3I", trial & 0xFFFFFFFF, trial >> 32, (3 << 16) | 4)
        pt = np.frombuffer(oracle.chacha20_xor(bytes(blob[32:32 + exp]), key32, 1, nonce), np.uint8)
        for part in range(2):  # K then V: [q][scale]
            off = part * (qb + 2)
            q_ref, sh_ref = _neon_group(x16[part], qmax)
            np.testing.assert_array_equal(pt[off:off + qb], q_ref, err_msg=f"trial {trial} part {part}")
            assert pt[off + qb:off + qb + 2].view(np.uint16)[0] == sh_ref.view(np.uint16), (trial, part)
