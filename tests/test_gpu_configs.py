"""The benchmark configurations at their full sizes, through the C-ABI, against the oracle and the reference
build: config 1 (64-page K8V4_ASYM), config 3 (256-page MLA 64x1x576), config 2's fidelity (256 pages,
32 queries per head) against the reference codec's own round trip, and config 4's 4,096-page prefix
(64 layers x 64 pages, shuffled block table, per-page layer ids and sequence nonces) for INT4_SYM and
K8V4_ASYM, every byte compared."""
from __future__ import annotations

import concurrent.futures as cf
import os

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
THREADS = min(16, os.cpu_count() or 1)


def _oracle_chunks(fn, n, chunk):
    """Run fn(a, b) over [0, n) in chunks on host threads (the oracle's ctypes calls release the GIL)."""
    with cf.ThreadPoolExecutor(THREADS) as ex:
        return list(ex.map(lambda a: fn(a, min(a + chunk, n)), range(0, n, chunk)))


def _round_trip_vs_oracle(oracle, shape, preset, rope_mode, pages, seed):
    from ztcp_b200 import capi, codec, workload

    k32, v32 = workload.kv_pages_np(pages, shape, seed=seed)
    kb = torch.from_numpy(k32).to(torch.bfloat16)
    vb = None if v32 is None else torch.from_numpy(v32).to(torch.bfloat16)
    m = workload.session_material(seed + 1)
    toks = workload.token_hashes(pages, seed + 2)
    g = capi.geometry(shape.num_tokens, shape.num_heads, shape.head_dim, shape.rope_dim, shape.mla)
    import ctypes as C

    payload = capi.load().ztcp_spec_payload_bytes(preset, rope_mode, C.byref(g), 0 if shape.mla else 1)
    keys = capi.keys(*m["key"], *m["mac_key"])
    blobs = torch.empty((pages, 48 + payload), dtype=torch.uint8, device=DEV)
    tok_d = torch.from_numpy(toks).to(DEV)
    codec.encode_pages(kb.to(DEV), None if vb is None else vb.to(DEV), tok_d, blobs, rope_dim=shape.rope_dim,
                       preset=preset, rope_mode=rope_mode, expected_payload_bytes=payload, tenant_id_hash=m["tenant"],
                       model_id_hash=m["model"], layer_id=m["layer"], head_group_id=m["head_group"],
                       base_sequence_nonce=m["base_seq"], keys=keys)
    kd = torch.empty(tuple(kb.shape), dtype=torch.float16, device=DEV)
    vd = None if vb is None else torch.empty_like(kd)
    st, fail = codec.decode_pages(blobs, tok_d, kd, vd, rope_dim=shape.rope_dim, is_mla=shape.mla,
                                  tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"], keys=keys)
    codec.raise_for_status(st, fail)
    got = blobs.cpu().numpy()
    k16 = kb.half().numpy()
    v16 = None if vb is None else vb.half().numpy()

    def enc(a, b):
        return helpers.oracle_encode(oracle, k16[a:b], None if v16 is None else v16[a:b], toks[a:b], shape.rope_dim,
                                     preset, rope_mode, payload, dict(m, base_seq=(m["base_seq"] + a) % 2**64))

    want = np.concatenate(_oracle_chunks(enc, pages, 16))
    np.testing.assert_array_equal(got, want)
    dims = (0, shape.num_tokens, shape.num_heads, shape.head_dim)

    def dec(a, b):
        return helpers.oracle_decode(oracle, want[a:b], toks[a:b], dims, shape.rope_dim, shape.mla, m)

    parts = _oracle_chunks(dec, pages, 16)
    assert all(p[3] == -1 for p in parts)
    np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), np.concatenate([p[0] for p in parts]))
    if vb is not None:
        np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), np.concatenate([p[1] for p in parts]))
    return kb, vb, kd, vd


def test_config1_k8v4_64_pages_bit_exact(oracle):
    """Config 1: 64 GQA pages, K8V4_ASYM + PRESERVE_FP8 (K NoPE INT8, V INT4), blobs and decoded pages
    bit-exact against the oracle (the reference's K8V4 peak path, bench_cold_page_pipeline.py:1041-1085)."""
    from ztcp_b200 import workload

    _round_trip_vs_oracle(oracle, workload.GQA, 2, 1, 64, 42)


def test_config3_mla_256_pages_bit_exact(oracle):
    """Config 3: 256 single-buffer MLA pages 64 x 1 x 576 with the 64 RoPE columns first, INT4_SYM +
    PRESERVE_FP8, and the softmax-weights cosine of 16 seed-99 query heads."""
    from ztcp_b200 import workload

    kb, _, kd, _ = _round_trip_vs_oracle(oracle, workload.MLA, 1, 1, 256, 42)
    cos = workload.attention_cosine(kb.float(), None, kd.cpu().float(), None, n_queries=16, seed=99)
    assert cos > 0.99, cos


def _reference_module():
    import build_ref

    try:
        return build_ref.load_module()
    except FileNotFoundError:
        return None


def test_config2_fidelity_equals_the_reference_codecs():
    """Config 2: config 0's 256 pages; the attention-output cosine (32 seed-99 queries per head, float64)
    of this codec's GPU round trip and of the reference codec's own CPU round trip (oracle/_ref: its peak
    egress on the same fp16 values, then its peak ingress) agree within 1e-4 -- and the decoded pages are
    identical, so they agree exactly."""
    from ztcp_b200 import capi, codec, workload

    ref = _reference_module()
    if ref is None:
        pytest.skip("the reference build (oracle/_ref) is absent")
    n = 256
    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=42)
    kb, vb = torch.from_numpy(k32).to(torch.bfloat16), torch.from_numpy(v32).to(torch.bfloat16)
    m = workload.session_material(7)
    toks = torch.from_numpy(workload.token_hashes(n, 11))
    key, mk = m["key"], m["mac_key"]
    # the reference's own round trip on the host
    blobs_ref = torch.empty((n, 98352), dtype=torch.uint8)
    ref.fused_encode_cold_pages_peak_into_cpu(kb.half(), vb.half(), toks, blobs_ref, 1, 1, 64, 98304, m["tenant"],
                                              m["model"], m["layer"], m["head_group"], m["base_seq"], key[0], key[1],
                                              mk[0], mk[1], key[2], key[3])
    kr, vr = torch.empty((n, 64, 8, 128), dtype=torch.float16), torch.empty((n, 64, 8, 128), dtype=torch.float16)
    ref.fused_decode_cold_pages_peak_into_cpu(blobs_ref, toks, kr, vr, 64, False, m["tenant"], m["model"], m["layer"],
                                              key[0], key[1], mk[0], mk[1], key[2], key[3])
    # this codec on the GPU, from the bf16 pages
    keys = capi.keys(*key, *mk)
    blobs = torch.empty((n, 98352), dtype=torch.uint8, device=DEV)
    td = toks.to(DEV)
    codec.encode_pages(kb.to(DEV), vb.to(DEV), td, blobs, rope_dim=64, preset=1, rope_mode=1,
                       expected_payload_bytes=98304, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                       layer_id=m["layer"], head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
    kd = torch.empty((n, 64, 8, 128), dtype=torch.float16, device=DEV)
    vd = torch.empty_like(kd)
    st, fail = codec.decode_pages(blobs, td, kd, vd, rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"],
                                  model_id_hash=m["model"], layer_id=m["layer"], keys=keys)
    codec.raise_for_status(st, fail)
    assert torch.equal(blobs.cpu(), blobs_ref)
    cos_ref = workload.attention_cosine(kb.float(), vb.float(), kr.float(), vr.float(), n_queries=32, seed=99)
    cos = workload.attention_cosine(kb.float(), vb.float(), kd.cpu().float(), vd.cpu().float(), n_queries=32, seed=99)
    assert abs(cos - cos_ref) <= 1e-4, (cos, cos_ref)
    assert cos > 0.99
    assert torch.equal(kd.cpu().view(torch.int16), kr.view(torch.int16))
    assert torch.equal(vd.cpu().view(torch.int16), vr.view(torch.int16))


@pytest.mark.parametrize("preset,payload", [(1, 98304), (2, 114688)], ids=["int4_sym", "k8v4_asym"])
def test_config4_prefix_4096_pages_bit_exact(oracle, preset, payload):
    """Config 4: a 4,096-page prefix (64 layers x 64 pages) in one launch per direction through a seeded
    shuffled block table over a 4,096-block pool, per-page layer ids (list position // 64) and sequence
    nonces; every blob and every decoded page equals the oracle's encode / decode of the addressed block
    with that page's layer id and nonce."""
    from ztcp_b200 import capi, codec, workload

    P = 4096
    kb, vb = workload.kv_pages_torch(P, workload.GQA, seed=4242, device=DEV)
    order = np.random.default_rng(4096).permutation(P).astype(np.int32)   # list position -> pool block
    layers = (np.arange(P) // 64).astype(np.int16)
    m = workload.session_material(31)
    seqs = np.arange(P, dtype=np.uint64) + np.uint64(m["base_seq"])   # wraps mod 2^64
    toks = workload.token_hashes(P, 4097)
    keys = capi.keys(*m["key"], *m["mac_key"])
    table = torch.from_numpy(order).to(DEV)
    td = torch.from_numpy(toks).to(DEV)
    ld = torch.from_numpy(layers).to(DEV)
    blobs = torch.empty((P, 48 + payload), dtype=torch.uint8, device=DEV)
    codec.encode_pages(kb, vb, td, blobs, rope_dim=64, preset=preset, rope_mode=1, expected_payload_bytes=payload,
                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=0, head_group_id=m["head_group"],
                       base_sequence_nonce=0, keys=keys, block_table=table,
                       sequence_nonces=torch.from_numpy(seqs.view(np.int64)).to(DEV), layer_ids=ld)
    kout = torch.zeros((P, 64, 8, 128), dtype=torch.float16, device=DEV)
    vout = torch.zeros_like(kout)
    st, fail = codec.decode_pages(blobs, td, kout, vout, rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"],
                                  model_id_hash=m["model"], layer_id=0, keys=keys, block_table=table, layer_ids=ld)
    codec.raise_for_status(st, fail)
    got = blobs.cpu().numpy()
    k16 = kb.half().cpu().numpy()[order]     # list order
    v16 = vb.half().cpu().numpy()[order]
    del kb, vb
    ko = kout.cpu().numpy().view(np.uint16)[order]
    vo = vout.cpu().numpy().view(np.uint16)[order]

    def check_layer(a, b):
        ml = dict(m, layer=int(layers[a]), base_seq=int(seqs[a]))
        want = helpers.oracle_encode(oracle, k16[a:b], v16[a:b], toks[a:b], 64, preset, 1, payload, ml)
        bad_blob = not np.array_equal(got[a:b], want)
        okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks[a:b], (0, 64, 8, 128), 64, False, ml)
        bad_dec = first != -1 or not np.array_equal(ko[a:b], okd) or not np.array_equal(vo[a:b], ovd)
        return a, bad_blob, bad_dec

    for a, bad_blob, bad_dec in _oracle_chunks(check_layer, P, 64):   # one chunk = one layer's 64 pages
        assert not bad_blob, f"blobs of layer {a // 64} differ from the oracle"
        assert not bad_dec, f"decoded pages of layer {a // 64} differ from the oracle"


@pytest.mark.parametrize("shape_name,preset", [("GQA", 1), ("GQA", 2), ("MLA", 1)])
def test_compiled_geometries_with_and_without_padding(oracle, shape_name, preset):
    """The compiled tile kernels (the benchmark geometries and formats) on their every path: whole tiles
    (the GQA egress stages its rows in shared memory by bulk copies), and a padded payload, whose last tile
    takes the general path inside the same kernel; fp16 and bf16 input with edge values, every byte against
    the oracle."""
    import ctypes as C

    from ztcp_b200 import capi, codec, workload

    shape = getattr(workload, shape_name)
    g = capi.geometry(shape.num_tokens, shape.num_heads, shape.head_dim, shape.rope_dim, shape.mla)
    base = capi.load().ztcp_spec_payload_bytes(preset, 1, C.byref(g), 0 if shape.mla else 1)
    rng = np.random.default_rng(606 + preset)
    edge = np.array([np.inf, -np.inf, 65504, -65504, 1e-7, -3e-6, 0.0, 7e4], dtype=np.float32)
    pages = 6
    for extra in (0, 16, 64):
        for bf16 in (False, True):
            k32, v32 = workload.kv_pages_np(pages, shape, seed=int(rng.integers(1 << 30)))
            for a in (k32, v32):
                if a is not None:
                    mask = rng.random(a.shape) < 0.01
                    a[mask] = rng.choice(edge, int(mask.sum()))
            with np.errstate(over="ignore"):
                if bf16:
                    kt = torch.from_numpy(k32).to(torch.bfloat16)
                    vt = None if v32 is None else torch.from_numpy(v32).to(torch.bfloat16)
                    k16, v16 = kt.half().numpy(), None if vt is None else vt.half().numpy()
                else:
                    k16, v16 = k32.astype(np.float16), None if v32 is None else v32.astype(np.float16)
                    kt, vt = torch.from_numpy(k16), None if v16 is None else torch.from_numpy(v16)
            m = workload.session_material(int(rng.integers(1 << 30)))
            toks = workload.token_hashes(pages, int(rng.integers(1 << 30)))
            exp = base + extra
            keys = capi.keys(*m["key"], *m["mac_key"])
            blobs = torch.empty((pages, 48 + exp), dtype=torch.uint8, device=DEV)
            codec.encode_pages(kt.to(DEV), None if vt is None else vt.to(DEV), torch.from_numpy(toks).to(DEV), blobs,
                               rope_dim=shape.rope_dim, preset=preset, rope_mode=1, expected_payload_bytes=exp,
                               tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                               head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
            want = helpers.oracle_encode(oracle, k16, v16, toks, shape.rope_dim, preset, 1, exp, m)
            tag = f"{shape_name} preset {preset} +{extra} bf16 {bf16}"
            np.testing.assert_array_equal(blobs.cpu().numpy(), want, err_msg=tag)
            kd = torch.empty(tuple(k16.shape), dtype=torch.float16, device=DEV)
            vd = None if v16 is None else torch.empty_like(kd)
            st, fail = codec.decode_pages(blobs, torch.from_numpy(toks).to(DEV), kd, vd, rope_dim=shape.rope_dim,
                                          is_mla=shape.mla, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                                          layer_id=m["layer"], keys=keys)
            codec.raise_for_status(st, fail)
            okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k16.shape, shape.rope_dim, shape.mla, m)
            assert first == -1, tag
            np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd, err_msg=tag)
            if vd is not None:
                np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd, err_msg=tag)
