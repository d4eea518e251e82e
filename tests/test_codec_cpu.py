"""Host-side checks of the batch API (no GPU): CPU tensors are refused before anything is packed, and stream
arguments resolve to raw handles."""
from __future__ import annotations

import pytest
import torch


def test_prepare_refuses_host_tensors():
    from ztcp_b200 import capi, codec

    k = torch.zeros((2, 64, 8, 128), dtype=torch.float16)
    toks = torch.zeros(2, dtype=torch.int64)
    blobs = torch.zeros((2, 98352), dtype=torch.uint8)
    keys = capi.keys(1, 2, 3, 4, 5, 6)
    with pytest.raises(RuntimeError, match="k_pages must be a CUDA tensor"):
        codec.prepare_encode(k, k, toks, blobs, rope_dim=64, preset=1, rope_mode=1, expected_payload_bytes=98304,
                             tenant_id_hash=1, model_id_hash=2, layer_id=3, head_group_id=4, base_sequence_nonce=5,
                             keys=keys)
    with pytest.raises(RuntimeError, match="cold_blobs must be a CUDA tensor"):
        codec.prepare_decode(blobs, toks, k, k, rope_dim=64, is_mla=False, tenant_id_hash=1, model_id_hash=2,
                             layer_id=3, keys=keys)


def test_stream_argument_forms():
    from ztcp_b200 import codec

    dev = torch.device("cuda", 0)
    assert codec._stream_arg(dev, 0) == 0
    assert codec._stream_arg(dev, 0x7F001234) == 0x7F001234

    class OtherDeviceStream:  # the attributes the codec reads from a torch.cuda.Stream
        device = torch.device("cuda", 1)
        cuda_stream = 99

    with pytest.raises(RuntimeError, match="stream must be on cuda:0"):
        codec._stream_arg(dev, OtherDeviceStream())


def test_prepared_call_owns_its_keys():
    from ztcp_b200 import capi, codec

    keys = capi.keys(1, 2, 3, 4, 5, 6)
    copy = codec._copy_keys(keys)
    keys.enc[0] = 0
    keys.mac[1] = 0
    assert list(copy.enc) == [1, 2, 3, 4] and list(copy.mac) == [5, 6]
