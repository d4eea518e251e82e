"""Wire-order egress of large batches (>= 1,024 pages): production launches in the blob's byte order with the tag
chains following segment by segment on a side stream.  Its blobs must equal, byte for byte, the single-pass
egress of the same pages (batches under the threshold, which the oracle pins everywhere else), for every
preset and RoPE mode, GQA and MLA, fp16 and bf16, with padded payloads and with block-table entries outside
the pool (those pages' blobs all zero)."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _encode(k, v, toks, blobs, payload, preset, rope_mode, rope_dim, m, keys, table=None, seqs=None):
    from ztcp_b200 import codec

    codec.encode_pages(k, v, toks, blobs, rope_dim=rope_dim, preset=preset, rope_mode=rope_mode,
                       expected_payload_bytes=payload, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                       layer_id=m["layer"], head_group_id=m["head_group"], base_sequence_nonce=0, keys=keys,
                       block_table=table, sequence_nonces=seqs, check_block_table=False)


@pytest.mark.parametrize("shape_name,preset,rope_mode,dtype,extra_pad", [
    ("GQA", 1, 1, torch.bfloat16, 0), ("GQA", 2, 1, torch.bfloat16, 0), ("GQA", 3, 2, torch.float16, 0),
    ("GQA", 1, 0, torch.float16, 64), ("MLA", 1, 1, torch.bfloat16, 0), ("MLA", 2, 2, torch.float16, 16)])
def test_wire_order_equals_single_pass(shape_name, preset, rope_mode, dtype, extra_pad):
    from ztcp_b200 import capi, workload

    shape = getattr(workload, shape_name)
    pool = 1100
    n = 1088                                   # >= 1,024 pages: wire order; 17 single-pass chunks of 64
    k, v = workload.kv_pages_torch(pool, shape, seed=71, dtype=dtype, device=DEV)
    g = capi.geometry(shape.num_tokens, shape.num_heads, shape.head_dim, shape.rope_dim, shape.mla)
    payload = capi.load().ztcp_spec_payload_bytes(preset, rope_mode, C.byref(g), 0 if shape.mla else 1) + extra_pad
    m = workload.session_material(72)
    keys = capi.keys(*m["key"], *m["mac_key"])
    rng = np.random.default_rng(73)
    table = rng.permutation(pool)[:n].astype(np.int32)
    table[[5, 700, n - 1]] = [pool, -3, pool + 9]  # outside the pool
    td = torch.from_numpy(table).to(DEV)
    toks = torch.from_numpy(workload.token_hashes(n, 74)).to(DEV)
    seqs = torch.from_numpy(rng.integers(-2**62, 2**62, n, dtype=np.int64)).to(DEV)
    whole = torch.full((n, 48 + payload), 0x5A, dtype=torch.uint8, device=DEV)
    _encode(k, v, toks, whole, payload, preset, rope_mode, shape.rope_dim, m, keys, td, seqs)
    parts = torch.full_like(whole, 0x33)
    for a in range(0, n, 64):
        _encode(k, v, toks[a:a + 64], parts[a:a + 64], payload, preset, rope_mode, shape.rope_dim, m, keys,
                td[a:a + 64], seqs[a:a + 64])
    torch.cuda.synchronize()
    bad = (td < 0) | (td >= pool)
    assert not whole[bad].any(), "pages outside the pool must be written as zeros"
    assert torch.equal(whole, parts)


def test_wire_order_then_decode_round_trip():
    """A 2,048-page wire-order egress decodes (one 2,048-page call) to the single-pass decode of its blobs."""
    from ztcp_b200 import capi, codec, workload

    n = 2048
    k, v = workload.kv_pages_torch(n, workload.GQA, seed=81, device=DEV)
    m = workload.session_material(82)
    keys = capi.keys(*m["key"], *m["mac_key"])
    toks = torch.from_numpy(workload.token_hashes(n, 83)).to(DEV)
    blobs = torch.empty((n, 98352), dtype=torch.uint8, device=DEV)
    codec.encode_pages(k, v, toks, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                       tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                       head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)
    ko = torch.empty((n, 64, 8, 128), dtype=torch.float16, device=DEV)
    vo = torch.empty_like(ko)
    st, fail = codec.decode_pages(blobs, toks, ko, vo, rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"],
                                  model_id_hash=m["model"], layer_id=m["layer"], keys=keys)
    codec.raise_for_status(st, fail)
    ko2, vo2 = torch.empty_like(ko), torch.empty_like(ko)
    for a in range(0, n, 256):
        st2, f2 = codec.decode_pages(blobs[a:a + 256], toks[a:a + 256], ko2[a:a + 256], vo2[a:a + 256], rope_dim=64,
                                     is_mla=False, tenant_id_hash=m["tenant"], model_id_hash=m["model"],
                                     layer_id=m["layer"], keys=keys)
        codec.raise_for_status(st2, f2)
    assert torch.equal(ko.view(torch.int16), ko2.view(torch.int16))
    assert torch.equal(vo.view(torch.int16), vo2.view(torch.int16))
    # single-pass egress of the same pages (chunks of 256 pages, sequence nonces continuing) gives the same blobs
    b2 = torch.empty_like(blobs)
    for a in range(0, n, 256):
        codec.encode_pages(k[a:a + 256], v[a:a + 256], toks[a:a + 256], b2[a:a + 256], rope_dim=64, preset=1,
                           rope_mode=1, expected_payload_bytes=98304, tenant_id_hash=m["tenant"],
                           model_id_hash=m["model"], layer_id=m["layer"], head_group_id=m["head_group"],
                           base_sequence_nonce=(m["base_seq"] + a) % 2**64, keys=keys)
    torch.cuda.synchronize()
    assert torch.equal(blobs, b2)


def test_captured_large_encode_takes_the_single_pass():
    """A 1,024-page encode captured into a CUDA graph stays on the capturing stream (single pass) and replays
    the same bytes as the eager call, which runs in wire order on the library's side streams."""
    from ztcp_b200 import capi, codec, workload

    n = 1024
    k, v = workload.kv_pages_torch(n, workload.GQA, seed=91, device=DEV)
    m = workload.session_material(92)
    keys = capi.keys(*m["key"], *m["mac_key"])
    toks = torch.from_numpy(workload.token_hashes(n, 93)).to(DEV)

    def enc(out):
        codec.encode_pages(k, v, toks, out, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                           tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                           head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"], keys=keys)

    eager = torch.empty((n, 98352), dtype=torch.uint8, device=DEV)
    enc(eager)
    replayed = torch.zeros_like(eager)
    s = torch.cuda.Stream(device=DEV)
    s.wait_stream(torch.cuda.current_stream(DEV))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        enc(replayed)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager, replayed)
    del g
