"""Peer gather (ztcp_b200.offload.gather / ztcp_gather): blobs encoded on two GPUs land back to back on one,
byte for byte.  Needs two GPUs; skipped otherwise."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gather_blobs_from_two_gpus():
    from ztcp_b200 import build, capi, codec, workload
    from ztcp_b200.offload import gather

    build.build()
    m = workload.session_material(5)
    keys = capi.keys(*m["key"], *m["mac_key"])
    parts = []
    for d in range(2):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            k, v = workload.kv_pages_torch(3 + d, workload.GQA, seed=40 + d, device=dev)
            toks = torch.from_numpy(workload.token_hashes(3 + d, 50 + d).view(np.int64)).to(dev)
            blobs = torch.empty((3 + d, 98352), dtype=torch.uint8, device=dev)
            codec.encode_pages(k, v, toks, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                               tenant_id_hash=m["tenant"], model_id_hash=m["model"], layer_id=m["layer"],
                               head_group_id=m["head_group"], base_sequence_nonce=m["base_seq"] + 100 * d, keys=keys)
        parts.append(blobs)
    out = gather(parts, "cuda:0")
    torch.cuda.synchronize("cuda:0")
    torch.cuda.synchronize("cuda:1")
    assert out.device == torch.device("cuda", 0) and out.shape == (7, 98352)
    np.testing.assert_array_equal(out.cpu().numpy(), torch.cat([p.cpu() for p in parts]).numpy())
