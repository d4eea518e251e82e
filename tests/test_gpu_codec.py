"""CUDA codec parity through the C-ABI: bit-exact wire bytes and decoded pages against the oracle and the
reference's golden vectors, at small sizes, at the benchmark configurations' full sizes, with block tables,
per-page metadata, misaligned blob strides, tampering and batch failure."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def ext():
    from ztcp_b200 import build, fused_ext

    build.build()
    assert torch.cuda.is_available()
    return fused_ext


def _keys(m):
    return dict(k0=m["key"][0], k1=m["key"][1], mk0=m["mac_key"][0], mk1=m["mac_key"][1], k2=m["key"][2],
                k3=m["key"][3])


def gpu_encode(ext, k, v, toks, rope, preset, rope_mode, exp, m):
    k = k.to(DEV)
    v = None if v is None else v.to(DEV)
    out = torch.empty((k.shape[0], 48 + exp), dtype=torch.uint8, device=DEV)
    ext.fused_encode_cold_pages_peak_into_cpu(k, v, torch.as_tensor(toks).to(DEV), out, preset, rope_mode, rope, exp,
                                              m["tenant"], m["model"], m["layer"], m["head_group"], m["base_seq"],
                                              **_keys(m))
    torch.cuda.synchronize()
    return out


def gpu_decode(ext, blobs, toks, shape4, rope, mla, m):
    k = torch.empty(shape4, dtype=torch.float16, device=DEV)
    v = None if mla else torch.empty(shape4, dtype=torch.float16, device=DEV)
    ext.fused_decode_cold_pages_peak_into_cpu(blobs.to(DEV), torch.as_tensor(toks).to(DEV), k, v, rope, mla,
                                              m["tenant"], m["model"], m["layer"], **_keys(m))
    return k, v


def test_chacha20_kats(ext):
    for v in helpers.load_json("kat_chacha20.json"):
        data = torch.tensor(list(bytes.fromhex(v["data"])), dtype=torch.uint8, device=DEV)
        key = torch.tensor(list(bytes.fromhex(v["key"])), dtype=torch.uint8)
        nonce = torch.tensor(list(bytes.fromhex(v["nonce"])), dtype=torch.uint8)
        out = ext.chacha20_rfc8439_xor_cpu(data, key, v["counter"], nonce)
        assert bytes(out.cpu().numpy()).hex() == v["out"]


def test_siphash_kats(ext):
    for v in helpers.load_json("kat_siphash.json"):
        k0, k1 = struct.unpack("<QQ", bytes.fromhex(v["key"]))
        data = torch.tensor(list(bytes.fromhex(v["data"])), dtype=torch.uint8, device=DEV)
        assert bytes(ext.siphash24_128_cpu(data, k0, k1).cpu().numpy()).hex() == v["tag"]


def test_codec_small_golden(ext):
    cases, arrays = helpers.small_cases()
    for c in cases:
        i = c["id"]
        shape = (-1, c["T"], c["H"], c["D"])
        k = torch.from_numpy(arrays[f"k{i}"].reshape(shape).view(np.float16).copy())
        v = None if c["mla"] else torch.from_numpy(arrays[f"v{i}"].reshape(shape).view(np.float16).copy())
        toks = torch.from_numpy(arrays[f"tok{i}"])
        blobs = gpu_encode(ext, k, v, toks, c["rope"], c["preset"], c["rope_mode"], c["expected_payload"],
                           c["material"])
        np.testing.assert_array_equal(blobs.cpu().numpy(), arrays[f"blobs{i}"], err_msg=f"encode {c}")
        kd, vd = gpu_decode(ext, torch.from_numpy(arrays[f"blobs{i}"]), toks, tuple(k.shape), c["rope"], c["mla"],
                            c["material"])
        np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), arrays[f"kdec{i}"].reshape(kd.shape),
                                      err_msg=f"decode {c}")
        if not c["mla"]:
            np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), arrays[f"vdec{i}"].reshape(vd.shape))


@pytest.mark.parametrize("case", helpers.load_json("codec_digests.json"), ids=lambda c: c["name"])
def test_full_size_digests_bf16_input(ext, case):
    kb, vb, k16, v16, m, toks, shape = helpers.full_case_inputs(case)
    blobs = gpu_encode(ext, kb, vb, torch.from_numpy(toks), shape.rope_dim, case["preset"], case["rope_mode"],
                       case["expected_payload"], m)
    assert blobs.shape[1] == case["blob_bytes"]
    assert helpers.sha(blobs.cpu().numpy()) == case["blobs_sha256"]
    # the fp16 path must produce the same bytes as bf16 rounded to fp16
    blobs16 = gpu_encode(ext, k16, v16, torch.from_numpy(toks), shape.rope_dim, case["preset"], case["rope_mode"],
                         case["expected_payload"], m)
    assert torch.equal(blobs, blobs16)
    kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks), tuple(k16.shape), shape.rope_dim, shape.mla, m)
    assert helpers.sha(kd.cpu().numpy()) == case["k_decoded_sha256"]
    if vd is not None:
        assert helpers.sha(vd.cpu().numpy()) == case["v_decoded_sha256"]


def test_config0_256_pages_bit_exact(ext, oracle):
    """Benchmark config 0 at full size: 256 GQA pages, INT4_SYM + PRESERVE_FP8, bf16 input."""
    from ztcp_b200 import workload

    k32, v32 = workload.kv_pages_np(256, workload.GQA, seed=42)
    kb, vb = torch.from_numpy(k32).to(torch.bfloat16), torch.from_numpy(v32).to(torch.bfloat16)
    m = workload.session_material(7)
    toks = workload.token_hashes(256, 11)
    exp = 98304
    blobs = gpu_encode(ext, kb, vb, torch.from_numpy(toks), 64, 1, 1, exp, m)
    want = helpers.oracle_encode(oracle, kb.half().numpy(), vb.half().numpy(), toks, 64, 1, 1, exp, m)
    np.testing.assert_array_equal(blobs.cpu().numpy(), want)
    kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks), tuple(kb.shape), 64, False, m)
    okd, ovd, st, first = helpers.oracle_decode(oracle, want, toks, tuple(kb.shape), 64, False, m)
    assert first == -1
    np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd)
    np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd)


@pytest.mark.parametrize("T,H,D,rope,extra", [(7, 3, 48, 16, 1), (100, 1, 64, 32, 3), (5, 2, 16, 16, 13),
                                               (130, 1, 32, 0, 6), (1, 1, 16, 0, 0)])
def test_ragged_geometry_and_misaligned_blobs(ext, oracle, T, H, D, rope, extra):
    """Tiles that do not divide the page, byte ranges off 64-byte blocks, and blob strides that are not
    multiples of 16 (or of 4) exercise the byte-granular paths."""
    from ztcp_b200 import workload

    rng = np.random.default_rng(T * 1000 + D)
    for preset in (1, 2, 3):
        for rope_mode in (0, 1, 2):
            for mla in (False, True):
                k = rng.standard_normal((3, T, H, D)).astype(np.float16)
                v = None if mla else rng.standard_normal((3, T, H, D)).astype(np.float16)
                m = workload.session_material(int(rng.integers(1 << 30)))
                toks = workload.token_hashes(3, int(rng.integers(1 << 30)))
                exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla) + extra
                blobs = gpu_encode(ext, torch.from_numpy(k), None if v is None else torch.from_numpy(v),
                                   torch.from_numpy(toks), rope, preset, rope_mode, exp, m)
                want = helpers.oracle_encode(oracle, k, v, toks, rope, preset, rope_mode, exp, m)
                np.testing.assert_array_equal(blobs.cpu().numpy(), want, err_msg=f"{preset} {rope_mode} {mla}")
                kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks), k.shape, rope, mla, m)
                okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k.shape, rope, mla, m)
                assert first == -1
                np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd)
                if not mla:
                    np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd)


def test_block_table_and_per_page_metadata(oracle):
    """Shuffled block table over a KV pool with per-page layer ids and sequence nonces (the offload sweep's
    addressing); each blob must equal the oracle's single-page encode of the addressed block."""
    from ztcp_b200 import capi, codec, workload

    rng = np.random.default_rng(4)
    pool = 40
    k32, v32 = workload.kv_pages_np(pool, workload.GQA, seed=8)
    kb = torch.from_numpy(k32).to(torch.bfloat16).to(DEV)
    vb = torch.from_numpy(v32).to(torch.bfloat16).to(DEV)
    n = 24
    table = rng.permutation(pool)[:n].astype(np.int32)
    layers = rng.integers(0, 64, n).astype(np.int16)
    seqs = rng.integers(0, 2**62, n).astype(np.int64)
    toks = workload.token_hashes(n, 3)
    m = workload.session_material(12)
    keys = capi.keys(*m["key"], *m["mac_key"])
    out = torch.empty((n, 98352), dtype=torch.uint8, device=DEV)
    codec.encode_pages(kb, vb, torch.from_numpy(toks).to(DEV), out, rope_dim=64, preset=1, rope_mode=1,
                       expected_payload_bytes=98304, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                       layer_id=0, head_group_id=m["head_group"], base_sequence_nonce=0, keys=keys,
                       block_table=torch.from_numpy(table).to(DEV), sequence_nonces=torch.from_numpy(seqs).to(DEV),
                       layer_ids=torch.from_numpy(layers).to(DEV))
    got = out.cpu().numpy()
    k16 = kb.half().cpu().numpy()
    v16 = vb.half().cpu().numpy()
    for i in range(n):
        mi = dict(m, layer=int(layers[i]), base_seq=int(seqs[i]))
        want = helpers.oracle_encode(oracle, k16[table[i]][None], v16[table[i]][None], toks[i:i + 1], 64, 1, 1, 98304,
                                     mi)
        np.testing.assert_array_equal(got[i], want[0], err_msg=f"page {i}")
    # decode back into a fresh pool through the same table, per-page expected layers
    kout = torch.zeros((pool, 64, 8, 128), dtype=torch.float16, device=DEV)
    vout = torch.zeros_like(kout)
    st, fail = codec.decode_pages(out, torch.from_numpy(toks).to(DEV), kout, vout, rope_dim=64, is_mla=False,
                                  tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=0, keys=keys,
                                  block_table=torch.from_numpy(table).to(DEV),
                                  layer_ids=torch.from_numpy(layers).to(DEV))
    codec.raise_for_status(st, fail)
    for i in range(n):
        mi = dict(m, layer=int(layers[i]))
        okd, ovd, _, first = helpers.oracle_decode(oracle, got[i:i + 1], toks[i:i + 1], (1, 64, 8, 128), 64, False, mi)
        assert first == -1
        np.testing.assert_array_equal(kout[table[i]].cpu().numpy().view(np.uint16), okd[0])
        np.testing.assert_array_equal(vout[table[i]].cpu().numpy().view(np.uint16), ovd[0])
    untouched = np.setdiff1d(np.arange(pool), table)
    assert not kout[torch.from_numpy(untouched).to(DEV).long()].any()


def _encoded_batch(ext, n=6):
    from ztcp_b200 import workload

    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=21)
    kb, vb = torch.from_numpy(k32).to(torch.bfloat16), torch.from_numpy(v32).to(torch.bfloat16)
    m = workload.session_material(22)
    toks = torch.from_numpy(workload.token_hashes(n, 23))
    return gpu_encode(ext, kb, vb, toks, 64, 1, 1, 98304, m), toks, m, kb


def _expect_batch_failure(ext, blobs, toks, m, msg, **over):
    mm = dict(m, **over)
    k = torch.full((blobs.shape[0], 64, 8, 128), 3.0, dtype=torch.float16, device=DEV)
    v = torch.full_like(k, 3.0)
    with pytest.raises(RuntimeError, match=msg):
        ext.fused_decode_cold_pages_peak_into_cpu(blobs, toks.to(DEV), k, v, 64, False, mm["tenant"], mm["model"],
                                                  mm["layer"], **_keys(mm))
    assert not k.any() and not v.any(), "a failed batch must zero every output page"


def test_tamper_and_aad_statuses(ext, oracle):
    blobs, toks, m, _ = _encoded_batch(ext)
    # reference tamper offsets for GQA INT4+FP8 (bench:318-377): scale byte, 16-byte NoPE swap, paired V flips
    vecs, gs, r, nd = 512, 16, 64, 64
    s_rope = 32 + vecs * r
    q_nope = s_rope + vecs * (r // gs) * 2
    q_v = q_nope + vecs * (nd // 2) + vecs * (nd // gs) * 2
    for mutate in (lambda b: b.__setitem__((3, s_rope), b[3, s_rope] ^ 1),
                   lambda b: b.__setitem__((1, slice(q_nope, q_nope + 32)),
                                           torch.cat([b[1, q_nope + 16:q_nope + 32], b[1, q_nope:q_nope + 16]])),
                   lambda b: (b.__setitem__((5, q_v), b[5, q_v] ^ 1), b.__setitem__((5, q_v + 16), b[5, q_v + 16] ^ 1)),
                   lambda b: b.__setitem__((0, 64), b[0, 64] ^ 1),
                   lambda b: b.__setitem__((2, -1), b[2, -1] ^ 0x80)):
        bad = blobs.clone()
        mutate(bad)
        _expect_batch_failure(ext, bad, toks, m, "KV_INTEGRITY_ERROR: Cold-page MAC verification failed")
    for over in (dict(tenant=m["tenant"] ^ 1), dict(model=m["model"] ^ 2), dict(layer=m["layer"] ^ 4)):
        _expect_batch_failure(ext, blobs, toks, m, "CROSS_TENANT_CONTAMINATION", **over)
    t2 = toks.clone()
    t2[4] ^= 1
    _expect_batch_failure(ext, blobs, t2, m, "CROSS_TENANT_CONTAMINATION")
    bad = blobs.clone()
    bad[2, 0] ^= 1
    _expect_batch_failure(ext, bad, toks, m, "Invalid cold-page header magic, version, or flags")
    # forged flags / truncated payload with valid tags -> the flags statuses (4, 5)
    forged = blobs.clone()
    forged[1, 3] = 0x04
    tag = oracle.siphash24_128(forged[1, :-16].cpu().numpy().tobytes(), *m["mac_key"])
    forged[1, -16:] = torch.tensor(list(tag), dtype=torch.uint8)
    _expect_batch_failure(ext, forged, toks, m, "Invalid cold-page header magic, version, or flags")
    # single-page API raises the single-page texts
    with pytest.raises(RuntimeError, match="Invalid cold-page header flags"):
        ext.fused_decode_cold_page_cpu(forged[1].contiguous(), 64, 8, 128, 64, False, m["tenant"], m["model"],
                                       m["layer"], int(toks[1]), **_keys(m))
    short = torch.cat([blobs[:, :32 + 1000], blobs[:, -16:]], dim=1).contiguous()
    for b in range(short.shape[0]):
        tag = oracle.siphash24_128(short[b, :-16].cpu().numpy().tobytes(), *m["mac_key"])
        short[b, -16:] = torch.tensor(list(tag), dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="payload truncated"):
        ext.fused_decode_cold_page_cpu(short[0].contiguous(), 64, 8, 128, 64, False, m["tenant"], m["model"],
                                       m["layer"], int(toks[0]), **_keys(m))


def test_host_placement_dropin(ext, oracle):
    """CPU tensors in and out (the reference wrapper's placement): staged through the GPU, same bytes."""
    from ztcp_b200 import workload

    k32, v32 = workload.kv_pages_np(3, workload.GQA, seed=31)
    k16 = torch.from_numpy(k32).half()
    v16 = torch.from_numpy(v32).half()
    m = workload.session_material(32)
    toks = torch.from_numpy(workload.token_hashes(3, 33))
    blobs = ext.fused_encode_cold_pages_batch_cpu(k16, v16, toks, 2, 1, 64, 114688, m["tenant"], m["model"],
                                                  m["layer"], m["head_group"], m["base_seq"], **_keys(m))
    assert blobs.device.type == "cpu"
    want = helpers.oracle_encode(oracle, k16.numpy(), v16.numpy(), toks.numpy(), 64, 2, 1, 114688, m)
    np.testing.assert_array_equal(blobs.numpy(), want)
    k, v = ext.fused_decode_cold_pages_batch_cpu(blobs, toks, 64, 8, 128, 64, False, m["tenant"], m["model"],
                                                 m["layer"], **_keys(m))
    okd, ovd, _, _ = helpers.oracle_decode(oracle, want, toks.numpy(), (3, 64, 8, 128), 64, False, m)
    np.testing.assert_array_equal(k.numpy().view(np.uint16), okd)
    one = ext.fused_encode_cold_page_cpu(k16[1], v16[1], 2, 1, 64, 114688, m["tenant"], m["model"], m["layer"],
                                         m["head_group"], int(toks[1]), m["base_seq"] + 1, **_keys(m))
    np.testing.assert_array_equal(one.numpy(), want[1])
    k1, v1 = ext.fused_decode_cold_page_cpu(one, 64, 8, 128, 64, False, m["tenant"], m["model"], m["layer"],
                                            int(toks[1]), **_keys(m))
    np.testing.assert_array_equal(k1.numpy().view(np.uint16), okd[1])


def test_fidelity_configs_2_and_3(ext):
    """Attention-output cosine (GQA, 32 queries/head, seed 99) and softmax-weights cosine (MLA, 16 query heads)."""
    from ztcp_b200 import workload

    k32, v32 = workload.kv_pages_np(16, workload.GQA, seed=42)
    kb, vb = torch.from_numpy(k32).to(torch.bfloat16), torch.from_numpy(v32).to(torch.bfloat16)
    m = workload.session_material(7)
    toks = torch.from_numpy(workload.token_hashes(16, 11))
    blobs = gpu_encode(ext, kb, vb, toks, 64, 1, 1, 98304, m)
    kd, vd = gpu_decode(ext, blobs, toks, tuple(kb.shape), 64, False, m)
    cos = helpers.attention_output_cosine(kb.float(), vb.float(), kd.cpu().float(), vd.cpu().float(), 32)
    assert cos > 0.99, cos
    k32, _ = workload.kv_pages_np(16, workload.MLA, seed=42)
    kb = torch.from_numpy(k32).to(torch.bfloat16)
    blobs = gpu_encode(ext, kb, None, toks, 64, 1, 1, 25088, m)
    kd, _ = gpu_decode(ext, blobs, toks, tuple(kb.shape), 64, True, m)
    cos = helpers.attention_output_cosine(kb.float(), None, kd.cpu().float(), None, 16)
    assert cos > 0.99, cos


def _tie_groups(qmax: int, n_groups: int, seed: int) -> np.ndarray:
    """fp16 groups whose largest |x| fixes the scale and whose other elements make x * (1/scale) round
    (in fp32) to an exact .5 tie while the unrounded product is not a tie: a fused multiply-add in place
    of the multiply then the rounding add would break those ties differently."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    out = []
    while len(out) < n_groups:
        amax = np.float16(rng.uniform(0.01, 300.0))
        scale = np.float16(f32(amax) * (f32(1.0) / f32(qmax)))
        if int(scale.view(np.uint16)) < 0x400:
            continue
        inv = f32(1.0) / f32(scale)
        cand = rng.uniform(-float(amax), float(amax), 4096).astype(np.float16)
        p32 = cand.astype(np.float32) * inv
        exact = cand.astype(np.float64) * np.float64(inv)
        frac = np.abs(p32 - np.trunc(p32))
        ties = cand[(frac == 0.5) & (exact != p32.astype(np.float64))]
        if len(ties) < 4:
            continue
        g = np.concatenate([[amax], ties[:15], np.zeros(15, np.float16)])[:16].astype(np.float16)
        out.append(rng.permutation(g))
    return np.stack(out)


@pytest.mark.parametrize("preset,rope_mode", [(1, 0), (3, 0)])
def test_rounding_ties_match_oracle(ext, oracle, preset, rope_mode):
    from ztcp_b200 import workload

    qmax = 7 if preset == 1 else 127
    T, H, D = 8, 4, 64
    groups = _tie_groups(qmax, 2 * T * H * D // 16, seed=preset)
    k = groups[: T * H * D // 16].reshape(1, T, H, D)
    v = groups[T * H * D // 16:].reshape(1, T, H, D)
    m = workload.session_material(77)
    toks = workload.token_hashes(1, 78)
    exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, 0, True)
    blobs = gpu_encode(ext, torch.from_numpy(k), torch.from_numpy(v), torch.from_numpy(toks), 0, preset, rope_mode,
                       exp, m)
    want = helpers.oracle_encode(oracle, k, v, toks, 0, preset, rope_mode, exp, m)
    np.testing.assert_array_equal(blobs.cpu().numpy(), want)


@pytest.mark.parametrize("T,H,D,rope", [(40, 2, 48, 16), (64, 8, 128, 64), (24, 4, 64, 0), (16, 8, 96, 32),
                                        (64, 1, 576, 64)])
def test_aligned_geometries_every_layout(ext, oracle, T, H, D, rope):
    """16-byte aligned blobs and regions on every preset x rope mode: tiles that do not divide the page,
    regions that start inside a 64-byte keystream block, bf16 and fp16 input, and edge values (inf, +-65504,
    values whose scale is subnormal) mixed into N(0,1) data."""
    from ztcp_b200 import workload

    rng = np.random.default_rng(T * 7 + D)
    edge = np.array([np.inf, -np.inf, 65504, -65504, 1e-7, -3e-6, 0.0, -0.0], dtype=np.float32)

    def page_values(shape):
        x = rng.standard_normal(shape).astype(np.float32)
        mask = rng.random(shape) < 0.03
        x[mask] = rng.choice(edge, int(mask.sum()))
        tiny = rng.random(shape[:3]) < 0.05  # whole rows of tiny values: subnormal scales
        x[tiny] *= 1e-6
        return x

    for preset in (1, 2, 3):
        for rope_mode in (0, 1, 2):
            for mla in ((True,) if D == 576 else (False, True)):
                for bf16 in (False, True):
                    k32 = page_values((3, T, H, D))
                    v32 = None if mla else page_values((3, T, H, D))
                    if bf16:
                        kt = torch.from_numpy(k32).to(torch.bfloat16)
                        vt = None if v32 is None else torch.from_numpy(v32).to(torch.bfloat16)
                        k16, v16 = kt.half().numpy(), None if vt is None else vt.half().numpy()
                    else:
                        k16, v16 = k32.astype(np.float16), None if v32 is None else v32.astype(np.float16)
                        kt, vt = torch.from_numpy(k16), None if v16 is None else torch.from_numpy(v16)
                    m = workload.session_material(int(rng.integers(1 << 30)))
                    toks = workload.token_hashes(3, int(rng.integers(1 << 30)))
                    exp = (oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla) + 15) // 16 * 16
                    blobs = gpu_encode(ext, kt, vt, torch.from_numpy(toks), rope, preset, rope_mode, exp, m)
                    want = helpers.oracle_encode(oracle, k16, v16, toks, rope, preset, rope_mode, exp, m)
                    tag = f"T{T} H{H} D{D} rope{rope} preset{preset} mode{rope_mode} mla{mla} bf16{bf16}"
                    np.testing.assert_array_equal(blobs.cpu().numpy(), want, err_msg=tag)
                    kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks), k16.shape, rope, mla, m)
                    okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k16.shape, rope, mla, m)
                    assert first == -1
                    np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd, err_msg=tag)
                    if not mla:
                        np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd, err_msg=tag)


@pytest.mark.parametrize("preset,rope_mode", [(1, 0), (3, 0), (2, 1)])
def test_bf16_groups_at_the_fp16_boundary(ext, oracle, preset, rope_mode):
    """bf16 input quantized without the fp16 round trip: groups whose amax sits just below, at and above
    the direct path's thresholds (2^-9 for INT4, 2^-5 for INT8) and that also hold values below fp16's
    normal range, values fp16 rounds (subnormal) and values past 65504 -- bytes equal the fp16 path's."""
    from ztcp_b200 import workload

    rng = np.random.default_rng(preset * 10 + rope_mode)
    T, H, D = 16, 2, 64
    n = 2 * T * H * D // 16
    amaxes = np.array([2.0**-9 * f for f in (0.99, 1.0, 1.01)] + [2.0**-5 * f for f in (0.99, 1.0, 1.01)]
                      + [1.0, 300.0, 6.5e4, 7.0e4], dtype=np.float32)
    tiny = np.array([2.0**-15, -2.0**-20, 3.1e-6, 2.0**-14, -6.0e-8, 0.0], dtype=np.float32)
    groups = []
    for i in range(n):
        g = rng.uniform(-1, 1, 16).astype(np.float32) * amaxes[i % len(amaxes)] * 0.9
        g[rng.integers(0, 16)] = amaxes[i % len(amaxes)] * (1 if i % 2 else -1)
        for j in rng.choice(16, 4, replace=False):
            g[j] = tiny[rng.integers(0, len(tiny))]
        groups.append(g)
    x = np.stack(groups).reshape(2, 1, T, H, D)
    kb = torch.from_numpy(x[0]).to(torch.bfloat16)
    vb = torch.from_numpy(x[1]).to(torch.bfloat16)
    m = workload.session_material(71)
    toks = workload.token_hashes(1, 72)
    exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, 16, True)
    blobs = gpu_encode(ext, kb, vb, torch.from_numpy(toks), 16, preset, rope_mode, exp, m)
    want = helpers.oracle_encode(oracle, kb.half().numpy(), vb.half().numpy(), toks, 16, preset, rope_mode, exp, m)
    np.testing.assert_array_equal(blobs.cpu().numpy(), want)


@pytest.mark.parametrize("mla", [False, True])
def test_neon_arithmetic_option(ext, oracle, mla):
    """The batch option that quantizes with the reference's ARM NEON fp16 arithmetic: bytes equal the
    oracle's NEON restatement (itself cross-checked against a numpy restatement; no ARM build runs
    here), on every preset x RoPE mode with edge values, fp16 and bf16 input; the standard ingress decodes
    the blobs (dequantization is the same in both arithmetics)."""
    from ztcp_b200 import capi, codec, workload

    rng = np.random.default_rng(17 + mla)
    T, H, D, rope = (16, 1, 96, 32) if mla else (16, 2, 64, 16)
    edge = np.array([np.inf, -np.inf, 65504, -65504, 1e-7, -3e-6, 0.0, 7e4], dtype=np.float32)
    for preset in (1, 2, 3):
        for rope_mode in (0, 1, 2):
            for bf16 in (False, True):
                x = (rng.standard_normal((2, 3, T, H, D)) * 10.0 ** rng.uniform(-4, 3)).astype(np.float32)
                mask = rng.random(x.shape) < 0.02
                x[mask] = rng.choice(edge, int(mask.sum()))
                if bf16:
                    kt = torch.from_numpy(x[0]).to(torch.bfloat16)
                    vt = None if mla else torch.from_numpy(x[1]).to(torch.bfloat16)
                    k16 = kt.half().numpy()
                    v16 = None if mla else vt.half().numpy()
                else:
                    with np.errstate(over="ignore"):  # 7e4 overflows to inf on purpose
                        k16 = x[0].astype(np.float16)
                        v16 = None if mla else x[1].astype(np.float16)
                    kt, vt = torch.from_numpy(k16), None if mla else torch.from_numpy(v16)
                m = workload.session_material(int(rng.integers(1 << 30)))
                toks = workload.token_hashes(3, int(rng.integers(1 << 30)))
                exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla)
                keys = capi.keys(*m["key"], *m["mac_key"])
                blobs = torch.empty((3, 48 + exp), dtype=torch.uint8, device=DEV)
                codec.encode_pages(kt.to(DEV), None if vt is None else vt.to(DEV), torch.from_numpy(toks).to(DEV),
                                   blobs, rope_dim=rope, preset=preset, rope_mode=rope_mode,
                                   expected_payload_bytes=exp, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                                   layer_id=m["layer"], head_group_id=m["head_group"],
                                   base_sequence_nonce=m["base_seq"], keys=keys, neon_arith=True)
                want = oracle.encode_batch(k16.view(np.uint16), None if v16 is None else v16.view(np.uint16), toks,
                                           rope_dim=rope, preset=preset, rope_mode=rope_mode, expected_payload=exp,
                                           tenant=m["tenant"], model=m["model"], layer=m["layer"],
                                           head_group=m["head_group"], base_seq=m["base_seq"], key=m["key"],
                                           mac_key=m["mac_key"], neon=True)
                tag = f"preset{preset} mode{rope_mode} mla{mla} bf16{bf16}"
                np.testing.assert_array_equal(blobs.cpu().numpy(), want, err_msg=tag)
                kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks), k16.shape, rope, mla, m)
                okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k16.shape, rope, mla, m)
                assert first == -1
                np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd, err_msg=tag)


def test_round_trip_replays_from_a_cuda_graph(ext, oracle):
    """The C-ABI neither allocates nor synchronizes, so an egress + ingress round trip can be captured in a
    CUDA graph and replayed (a launch-bound caller's way to cut host time); replays write the oracle's bytes."""
    from ztcp_b200 import capi, codec, workload

    n = 16
    m = workload.session_material(91)
    k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=92)
    k = torch.from_numpy(k32).to(torch.bfloat16).to(DEV)
    v = torch.from_numpy(v32).to(torch.bfloat16).to(DEV)
    toks_np = workload.token_hashes(n, 93)
    toks = torch.from_numpy(toks_np.view(np.int64)).to(DEV)
    keys = capi.keys(*m["key"], *m["mac_key"])
    blobs = torch.zeros((n, 98352), dtype=torch.uint8, device=DEV)
    ko = torch.zeros((n, 64, 8, 128), dtype=torch.float16, device=DEV)
    vo = torch.zeros_like(ko)
    st = torch.empty(n, dtype=torch.int32, device=DEV)
    fl = torch.empty(1, dtype=torch.int32, device=DEV)

    def round_trip():
        codec.encode_pages(k, v, toks, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                           tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                           head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
        codec.decode_pages(blobs, toks, ko, vo, rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"],
                           model_id_hash=m["model"], layer_id=m["layer"], keys=keys, status=st, any_fail=fl)

    side = torch.cuda.Stream(DEV)
    with torch.cuda.stream(side):
        round_trip()  # first launches (per-device kernel attributes) outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        round_trip()
    want = helpers.oracle_encode(oracle, k.cpu().half().numpy(), v.cpu().half().numpy(), toks_np, 64, 1, 1, 98304, m)
    okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks_np, (n, 64, 8, 128), 64, False, m)
    assert first == -1
    for _ in range(3):
        blobs.zero_()
        ko.zero_()
        vo.zero_()
        g.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(blobs.cpu().numpy(), want)
        assert int(fl.item()) == 0
        np.testing.assert_array_equal(ko.cpu().numpy().view(np.uint16), okd)
        np.testing.assert_array_equal(vo.cpu().numpy().view(np.uint16), ovd)
    del g


def test_seeded_random_sweep(ext, oracle):
    """120 seeded random configurations -- geometry (tokens, heads, head_dim up to 576, RoPE width), preset,
    RoPE mode, GQA or single-buffer MLA, fp16 or bf16 input, page count, payload padding (so blob strides
    of every alignment) and magnitudes from 1e-6 to 1e4 with edge values -- each encoded and decoded on the
    GPU and compared byte for byte with the oracle."""
    from ztcp_b200 import capi, codec, workload

    rng = np.random.default_rng(20261202)
    edge = np.array([np.inf, -np.inf, 65504, -65504, 1e-7, -3e-6, 0.0, 7e4], dtype=np.float32)
    for case in range(120):
        D = int(rng.choice([16, 32, 48, 64, 96, 128, 192, 256, 576]))
        T, H = int(rng.integers(1, 65)), int(rng.integers(1, 9 if D <= 128 else 3))
        rope = int(rng.integers(0, D // 16 + 1)) * 16
        rope_mode = int(rng.integers(0, 3)) if rope > 0 else 0
        preset, mla = int(rng.integers(1, 4)), bool(rng.random() < 0.3)
        bf16, n, extra = bool(rng.random() < 0.5), int(rng.integers(1, 5)), int(rng.integers(0, 41))
        x = (rng.standard_normal((2, n, T, H, D)) * 10.0 ** rng.uniform(-6, 4)).astype(np.float32)
        mask = rng.random(x.shape) < 0.02
        x[mask] = rng.choice(edge, int(mask.sum()))
        with np.errstate(over="ignore"):
            if bf16:
                kt = torch.from_numpy(x[0]).to(torch.bfloat16)
                vt = None if mla else torch.from_numpy(x[1]).to(torch.bfloat16)
                k16, v16 = kt.half().numpy(), None if mla else vt.half().numpy()
            else:
                k16, v16 = x[0].astype(np.float16), None if mla else x[1].astype(np.float16)
                kt, vt = torch.from_numpy(k16), None if mla else torch.from_numpy(v16)
        m = workload.session_material(int(rng.integers(1 << 30)))
        toks = workload.token_hashes(n, int(rng.integers(1 << 30)))
        exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla) + extra
        keys = capi.keys(*m["key"], *m["mac_key"])
        tag = f"case {case}: T{T} H{H} D{D} rope{rope} preset{preset} mode{rope_mode} mla{mla} bf16{bf16} n{n} +{extra}"
        blobs = torch.empty((n, 48 + exp), dtype=torch.uint8, device=DEV)
        codec.encode_pages(kt.to(DEV), None if vt is None else vt.to(DEV), torch.from_numpy(toks.view(np.int64)).to(DEV),
                           blobs, rope_dim=rope, preset=preset, rope_mode=rope_mode, expected_payload_bytes=exp,
                           tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                           head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
        want = helpers.oracle_encode(oracle, k16, v16, toks, rope, preset, rope_mode, exp, m)
        np.testing.assert_array_equal(blobs.cpu().numpy(), want, err_msg=tag)
        kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks.view(np.int64)), k16.shape, rope, mla, m)
        okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k16.shape, rope, mla, m)
        assert first == -1, tag
        np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd, err_msg=tag)
        if not mla:
            np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd, err_msg=tag)


def test_neon_option_random_sweep(ext, oracle):
    """The NEON-arithmetic egress option on 40 seeded random configurations (geometry, preset, RoPE mode,
    GQA/MLA, fp16/bf16, padding, magnitudes 1e-6 to 1e4 with edge values): bytes equal the oracle's NEON
    restatement and the blobs decode to the oracle's pages."""
    from ztcp_b200 import capi, codec, workload

    rng = np.random.default_rng(4242)
    edge = np.array([np.inf, -np.inf, 65504, -65504, 1e-7, -3e-6, 0.0, 7e4], dtype=np.float32)
    for case in range(40):
        D = int(rng.choice([16, 32, 64, 96, 128, 192, 576]))
        T, H = int(rng.integers(1, 49)), int(rng.integers(1, 9 if D <= 128 else 3))
        rope = int(rng.integers(0, D // 16 + 1)) * 16
        rope_mode = int(rng.integers(0, 3)) if rope > 0 else 0
        preset, mla = int(rng.integers(1, 4)), bool(rng.random() < 0.3)
        bf16, n, extra = bool(rng.random() < 0.5), int(rng.integers(1, 4)), int(rng.integers(0, 33))
        x = (rng.standard_normal((2, n, T, H, D)) * 10.0 ** rng.uniform(-6, 4)).astype(np.float32)
        mask = rng.random(x.shape) < 0.02
        x[mask] = rng.choice(edge, int(mask.sum()))
        with np.errstate(over="ignore"):
            if bf16:
                kt = torch.from_numpy(x[0]).to(torch.bfloat16)
                vt = None if mla else torch.from_numpy(x[1]).to(torch.bfloat16)
                k16, v16 = kt.half().numpy(), None if mla else vt.half().numpy()
            else:
                k16, v16 = x[0].astype(np.float16), None if mla else x[1].astype(np.float16)
                kt, vt = torch.from_numpy(k16), None if mla else torch.from_numpy(v16)
        m = workload.session_material(int(rng.integers(1 << 30)))
        toks = workload.token_hashes(n, int(rng.integers(1 << 30)))
        exp = oracle.spec_payload_bytes(preset, rope_mode, T * H, D, rope, not mla) + extra
        tag = f"case {case}: T{T} H{H} D{D} rope{rope} preset{preset} mode{rope_mode} mla{mla} bf16{bf16} n{n} +{extra}"
        blobs = torch.empty((n, 48 + exp), dtype=torch.uint8, device=DEV)
        codec.encode_pages(kt.to(DEV), None if vt is None else vt.to(DEV), torch.from_numpy(toks.view(np.int64)).to(DEV),
                           blobs, rope_dim=rope, preset=preset, rope_mode=rope_mode, expected_payload_bytes=exp,
                           tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                           head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"],
                           keys=capi.keys(*m["key"], *m["mac_key"]), neon_arith=True)
        want = oracle.encode_batch(k16.view(np.uint16), None if v16 is None else v16.view(np.uint16), toks,
                                   rope_dim=rope, preset=preset, rope_mode=rope_mode, expected_payload=exp,
                                   tenant=m["tenant"], model=m["model"], layer=m["layer"], head_group=m["head_group"],
                                   base_seq=m["base_seq"], key=m["key"], mac_key=m["mac_key"], neon=True)
        np.testing.assert_array_equal(blobs.cpu().numpy(), want, err_msg=tag)
        kd, vd = gpu_decode(ext, blobs, torch.from_numpy(toks.view(np.int64)), k16.shape, rope, mla, m)
        okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks, k16.shape, rope, mla, m)
        assert first == -1, tag
        np.testing.assert_array_equal(kd.cpu().numpy().view(np.uint16), okd, err_msg=tag)
        if not mla:
            np.testing.assert_array_equal(vd.cpu().numpy().view(np.uint16), ovd, err_msg=tag)
