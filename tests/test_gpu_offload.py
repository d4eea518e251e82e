"""Offload pipeline (ztcp_b200.offload): egress from host memory to pinned host blobs and ingress back, several
batches in flight on the pipeline's slots; bytes equal the oracle's, a tampered batch raises on wait() with
its outputs zeroed while the other batches decode."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import helpers

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_host_round_trips_in_flight(oracle):
    from ztcp_b200 import build, capi, workload
    from ztcp_b200.offload import OffloadPipeline

    build.build()
    m = workload.session_material(31)
    keys = capi.keys(*m["key"], *m["mac_key"])
    pipe = OffloadPipeline(DEV, slots=4)
    B, n = 5, 8
    ins, outs, tickets = [], [], []
    for b in range(B):
        k32, v32 = workload.kv_pages_np(n, workload.GQA, seed=100 + b)
        k = torch.from_numpy(k32).to(torch.bfloat16).pin_memory()
        v = torch.from_numpy(v32).to(torch.bfloat16).pin_memory()
        toks = torch.from_numpy(workload.token_hashes(n, 200 + b).view(np.int64)).pin_memory()
        blobs = torch.empty((n, 98352), dtype=torch.uint8).pin_memory()
        t = pipe.egress(k, v, toks, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                        tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                        head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"] + 1000 * b, keys=keys)
        if b == 3:  # tamper with batch 3 on the host once its blobs are down, before it is uploaded again
            t.wait()
            blobs[1, 4000] ^= 0x40
        ko = torch.empty((n, 64, 8, 128), dtype=torch.float16).pin_memory()
        vo = torch.empty_like(ko).pin_memory()
        tickets.append((t, pipe.ingress(blobs, toks, ko, vo, rope_dim=64, is_mla=False, tenant_id_hash=m["tenant"],
                                        model_id_hash=m["model"], layer_id=m["layer"], keys=keys, after=t)))
        ins.append((k, v, toks, b))
        outs.append((blobs, ko, vo))
    for (te, ti), (k, v, toks, b), (blobs, ko, vo) in zip(tickets, ins, outs):
        te.wait()
        mb = dict(m, base_seq=m["base_seq"] + 1000 * b)
        want = helpers.oracle_encode(oracle, k.half().numpy(), v.half().numpy(), toks.numpy().view(np.uint64), 64, 1, 1,
                                     98304, mb)
        if b == 3:
            with pytest.raises(RuntimeError, match="KV_INTEGRITY_ERROR: Cold-page MAC verification failed"):
                ti.wait()
            assert not ko.any() and not vo.any()
            want[1, 4000] ^= 0x40
            np.testing.assert_array_equal(blobs.numpy(), want)
            continue
        ti.wait()
        np.testing.assert_array_equal(blobs.numpy(), want)
        okd, ovd, _, first = helpers.oracle_decode(oracle, want, toks.numpy().view(np.uint64), (n, 64, 8, 128), 64,
                                                   False, mb)
        assert first == -1
        np.testing.assert_array_equal(ko.numpy().view(np.uint16), okd)
        np.testing.assert_array_equal(vo.numpy().view(np.uint16), ovd)
    pipe.synchronize()
