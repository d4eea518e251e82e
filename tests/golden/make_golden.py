"""Generate the golden vectors under tests/golden/ (run where the reference is present).

Sources of truth, all taken from the reference itself:
  * ChaCha20: the reference's Python RFC 8439 block function
    (research/baseline_codec/fused_quant_crypto.py:662-697) and its compiled
    codec's chacha20_rfc8439_xor_cpu (csrc:2499-2523); every vector is also
    cross-checked against the `cryptography` package's ChaCha20.
  * SipHash-2-4-128: the reference's Python siphash24_128 (fused_quant_crypto.py:700-752)
    and the compiled siphash24_128_cpu (csrc:2525-2538).
  * Codec blobs and decoded pages: the reference codec compiled from its own
    source by oracle/build_ref.py (fused_encode_cold_pages_peak_into_cpu and
    fused_decode_cold_pages_peak_into_cpu).

Outputs: kat_chacha20.json, kat_siphash.json, codec_small.npz + codec_small.json
(small pages, every preset x rope mode, GQA and MLA, edge values), and
codec_digests.json (SHA-256 of full-size blobs / decoded pages for the
benchmark configurations; inputs are regenerated from seeds by
ztcp_b200.workload.kv_pages_np).

Usage: python tests/golden/make_golden.py [--reference-root /path/to/reference]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "vlx-tee_b200"))

M64 = (1 << 64) - 1


def _cryptography_chacha(key: bytes, counter: int, nonce: bytes, data: bytes) -> bytes:
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms

    c = Cipher(algorithms.ChaCha20(key, struct.pack("<I", counter) + nonce), mode=None).encryptor()
    return c.update(data) + c.finalize()


def make_kats(fq, ref, torch):
    rng = np.random.default_rng(2026)
    chacha = []
    for length in [0, 1, 15, 63, 64, 65, 127, 128, 255, 256, 257, 1000, 4096, 5000]:
        key = rng.integers(0, 256, 32, dtype=np.uint8).tobytes()
        nonce = rng.integers(0, 256, 12, dtype=np.uint8).tobytes()
        counter = int(rng.choice([0, 1, 7, 0xFFFFFFF0]))
        data = rng.integers(0, 256, length, dtype=np.uint8).tobytes()
        # reference Python block function, keystream assembled per 64-byte block
        ks = b"".join(fq.chacha20_rfc8439_block(key, (counter + i) & 0xFFFFFFFF, nonce)
                      for i in range((length + 63) // 64))
        out_py = bytes(a ^ b for a, b in zip(data, ks))
        out_cpp = ref.chacha20_rfc8439_xor_cpu(torch.frombuffer(bytearray(data), dtype=torch.uint8) if length else
                                               torch.zeros(0, dtype=torch.uint8),
                                               torch.frombuffer(bytearray(key), dtype=torch.uint8), counter,
                                               torch.frombuffer(bytearray(nonce), dtype=torch.uint8)).numpy().tobytes()
        assert out_py == out_cpp, "reference Python and C++ ChaCha20 disagree"
        if counter + (length + 63) // 64 <= 0xFFFFFFFF:  # `cryptography` carries the counter into the nonce
            assert out_py == _cryptography_chacha(key, counter, nonce, data), "cryptography ChaCha20 disagrees"
        chacha.append({"key": key.hex(), "counter": counter, "nonce": nonce.hex(), "data": data.hex(),
                       "out": out_py.hex()})
    sip = []
    for length in list(range(0, 65)) + [100, 1000, 12345]:
        k = rng.integers(0, 256, 16, dtype=np.uint8).tobytes()
        data = rng.integers(0, 256, length, dtype=np.uint8).tobytes()
        tag_py = fq.siphash24_128(k, data)
        k0, k1 = struct.unpack("<QQ", k)
        tag_cpp = ref.siphash24_128_cpu(torch.frombuffer(bytearray(data), dtype=torch.uint8) if length else
                                        torch.zeros(0, dtype=torch.uint8), k0, k1).numpy().tobytes()
        assert tag_py == tag_cpp, "reference Python and C++ SipHash disagree"
        sip.append({"key": k.hex(), "data": data.hex(), "tag": tag_py.hex()})
    with open(os.path.join(HERE, "kat_chacha20.json"), "w") as f:
        json.dump(chacha, f, indent=0)
    with open(os.path.join(HERE, "kat_siphash.json"), "w") as f:
        json.dump(sip, f, indent=0)


def ref_encode(ref, torch, k16, v16, toks, rope, preset, rmode, exp, m):
    B = k16.shape[0]
    out = torch.zeros((B, 48 + exp), dtype=torch.uint8)
    ref.fused_encode_cold_pages_peak_into_cpu(
        torch.from_numpy(k16.copy()), None if v16 is None else torch.from_numpy(v16.copy()),
        torch.from_numpy(toks.copy()), out, preset, rmode, rope, exp, m["tenant"], m["model"], m["layer"],
        m["head_group"], m["base_seq"], m["key"][0], m["key"][1], m["mac_key"][0], m["mac_key"][1],
        m["key"][2], m["key"][3])
    return out.numpy()


def ref_decode(ref, torch, blobs, toks, shape4, rope, mla, m):
    k = torch.zeros(shape4, dtype=torch.float16)
    v = None if mla else torch.zeros(shape4, dtype=torch.float16)
    ref.fused_decode_cold_pages_peak_into_cpu(
        torch.from_numpy(blobs.copy()), torch.from_numpy(toks.copy()), k, v, rope, mla, m["tenant"], m["model"],
        m["layer"], m["key"][0], m["key"][1], m["mac_key"][0], m["mac_key"][1], m["key"][2], m["key"][3])
    return k.numpy(), None if v is None else v.numpy()


def make_codec_small(ref, torch):
    from ztcp_b200 import workload

    import ztcp_oracle as zo

    rng = np.random.default_rng(99)
    arrays, cases = {}, []
    geoms = [(2, 2, 32, 16), (3, 1, 64, 32), (1, 1, 16, 0), (2, 1, 48, 48)]
    edge_pool = np.array([0.0, -0.0, 1e-7, -2e-6, 5e-6, np.inf, -np.inf, 65504, -65504, 1.0, -7.0, 0.5],
                         np.float32)
    idx = 0
    for (T, H, D, rope) in geoms:
        for preset in (1, 2, 3):
            for rmode in (0, 1, 2):
                for mla in (False, True):
                    for kind in ("randn", "edge"):
                        B = 2
                        if kind == "randn":
                            k = (rng.standard_normal((B, T, H, D)) * rng.choice([0.02, 1.0, 40.0])).astype(np.float16)
                            v = rng.standard_normal((B, T, H, D)).astype(np.float16)
                        else:
                            k = rng.choice(edge_pool, (B, T, H, D)).astype(np.float16)
                            v = rng.choice(edge_pool, (B, T, H, D)).astype(np.float16)
                            k[0, 0, 0, :16] = 0.0
                            v[0, 0, 0, :16] = 1e-7
                        if mla:
                            v = None
                        m = workload.session_material(seed=1000 + idx)
                        toks = workload.token_hashes(B, seed=2000 + idx)
                        extra = 0 if idx % 3 else 20
                        exp = zo.spec_payload_bytes(preset, rmode, T * H, D, rope, not mla) + extra
                        blobs = ref_encode(ref, torch, k, v, toks, rope, preset, rmode, exp, m)
                        kd, vd = ref_decode(ref, torch, blobs, toks, (B, T, H, D), rope, mla, m)
                        arrays[f"k{idx}"] = k.view(np.uint16)
                        if v is not None:
                            arrays[f"v{idx}"] = v.view(np.uint16)
                        arrays[f"blobs{idx}"] = blobs
                        arrays[f"kdec{idx}"] = kd.view(np.uint16)
                        if vd is not None:
                            arrays[f"vdec{idx}"] = vd.view(np.uint16)
                        arrays[f"tok{idx}"] = toks
                        cases.append({"id": idx, "T": T, "H": H, "D": D, "rope": rope, "preset": preset,
                                      "rope_mode": rmode, "mla": mla, "kind": kind, "expected_payload": exp,
                                      "material": m})
                        idx += 1
    np.savez_compressed(os.path.join(HERE, "codec_small.npz"), **arrays)
    with open(os.path.join(HERE, "codec_small.json"), "w") as f:
        json.dump(cases, f, indent=0)


FULL_CASES = [
    # name, shape, preset, rope_mode, pages, seed
    ("gqa_int4_fp8", "GQA", 1, 1, 8, 42),
    ("gqa_k8v4_fp8", "GQA", 2, 1, 4, 43),
    ("gqa_int4_quantall", "GQA", 1, 0, 4, 44),
    ("gqa_fp8only_raw", "GQA", 3, 2, 2, 45),
    ("mla_int4_fp8", "MLA", 1, 1, 8, 46),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_digests(ref, torch):
    from ztcp_b200 import workload

    out = []
    for name, shape_name, preset, rmode, n, seed in FULL_CASES:
        shape = getattr(workload, shape_name)
        k32, v32 = workload.kv_pages_np(n, shape, seed=seed)
        # bf16 inputs, handed to the reference as bf16.half() (its codec accepts fp16 only)
        kb = torch.from_numpy(k32).to(torch.bfloat16)
        vb = None if v32 is None else torch.from_numpy(v32).to(torch.bfloat16)
        k16 = kb.half().numpy()
        v16 = None if vb is None else vb.half().numpy()
        m = workload.session_material(seed=seed)
        toks = workload.token_hashes(n, seed=seed + 1)
        from ztcp_b200.cold_page_spec import ColdPageGeometry, QuantPreset, RoPEMode

        geo = ColdPageGeometry(shape.num_tokens, shape.num_heads, shape.head_dim, shape.rope_dim,
                               is_mla_single_buffer=shape.mla)
        exp = geo.payload_bytes(QuantPreset(preset), RoPEMode(rmode))
        blobs = ref_encode(ref, torch, k16, v16, toks, shape.rope_dim, preset, rmode, exp, m)
        kd, vd = ref_decode(ref, torch, blobs, toks, k16.shape, shape.rope_dim, shape.mla, m)
        out.append({"name": name, "shape": shape_name, "preset": preset, "rope_mode": rmode, "pages": n,
                    "seed": seed, "expected_payload": exp, "blob_bytes": int(blobs.shape[1]),
                    "input_bf16_sha256": sha(kb.view(torch.int16).numpy()) + ("" if vb is None else
                                                                              sha(vb.view(torch.int16).numpy())),
                    "blobs_sha256": sha(blobs), "k_decoded_sha256": sha(kd),
                    "v_decoded_sha256": None if vd is None else sha(vd),
                    "first_blob_head_hex": blobs[0, :64].tobytes().hex(),
                    "first_tag_hex": blobs[0, -16:].tobytes().hex()})
    with open(os.path.join(HERE, "codec_digests.json"), "w") as f:
        json.dump(out, f, indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=os.environ.get(
        "ZTCP_REFERENCE_ROOT", os.path.join(os.path.dirname(REPO), "reference")))
    args = ap.parse_args()
    import torch

    import build_ref

    sys.path.insert(0, args.reference_root)
    import research.baseline_codec.fused_quant_crypto as fq

    build_ref.build(args.reference_root)
    ref = build_ref.load_module()
    make_kats(fq, ref, torch)
    make_codec_small(ref, torch)
    make_digests(ref, torch)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
