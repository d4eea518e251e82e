"""The drop-in boundary, checked against the reference's own wrapper (CPU, where the reference source is
present): NativeCppFusedColdPageCodec drives every `_ext` entry point through its real keyring flow; each
call it makes must bind to the ztcp_b200.fused_ext function of the same name."""
from __future__ import annotations

import inspect
import os
import sys

import pytest
import torch

REF_ROOT = os.environ.get("ZTCP_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                       "reference"))


class _Recorder:
    """Forwards to the reference codec module and records (name, args, kwargs)."""

    def __init__(self, mod):
        self._mod = mod
        self.calls = []

    def __getattr__(self, name):
        fn = getattr(self._mod, name)

        def call(*args, **kwargs):
            self.calls.append((name, args, kwargs))
            return fn(*args, **kwargs)

        return call


@pytest.fixture(scope="module")
def reference():
    if not os.path.isdir(os.path.join(REF_ROOT, "research", "baseline_codec")):
        pytest.skip("reference source not present")
    import build_ref

    try:
        mod = build_ref.load_module()
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")
    sys.path.insert(0, REF_ROOT)
    from research.baseline_codec import cold_page_spec, fused_quant_crypto, native_fused_codec

    return mod, cold_page_spec, fused_quant_crypto, native_fused_codec


def test_wrapper_calls_bind_to_fused_ext(reference):
    from ztcp_b200 import fused_ext

    mod, spec, fq, nfc = reference
    rec = _Recorder(mod)
    geom = spec.ColdPageGeometry(num_tokens=4, num_kv_heads=2, head_dim=32, rope_dim=16)
    ring = fq.EphemeralSessionKeyRing(deployment_pepper=b"p" * 32)
    codec = nfc.NativeCppFusedColdPageCodec.__new__(nfc.NativeCppFusedColdPageCodec)
    codec.geometry, codec.keyring, codec._ext = geom, ring, rec

    g = torch.Generator().manual_seed(3)
    k = torch.randn((3, 4, 2, 32), generator=g).half()
    v = torch.randn((3, 4, 2, 32), generator=g).half()
    toks = torch.tensor([11, 12, 13], dtype=torch.int64)
    aad = spec.ColdPageAAD(spec.hash32("t"), spec.hash32("m"), 5, 11, ring.next_sequence_nonce("t", "s", 8),
                           spec.QuantPreset.INT4_SYM, spec.RoPEMode.PRESERVE_FP8)
    blob_bytes = geom.cold_blob_bytes(aad.preset, aad.rope_mode)

    out = torch.zeros((3, blob_bytes), dtype=torch.uint8)
    codec.encode_cold_pages_peak_into(k, v, toks, out, "t", "s", aad)
    import dataclasses

    toks2 = torch.tensor([14, 15, 16], dtype=torch.int64)  # distinct slots: the keyring tracks versions per slot
    blobs = codec.encode_cold_pages_batch_tensor(k, v, toks2, "t", "s",
                                                 dataclasses.replace(aad, sequence_nonce=aad.sequence_nonce + 3))
    one = codec.encode_cold_page_tensor(k[0], v[0], "t", "s",
                                        dataclasses.replace(aad, sequence_nonce=aad.sequence_nonce + 6,
                                                            page_token_hash=21))
    codec.decode_cold_page_tensor(one, "t", "s", "m", 5, 21)
    codec.decode_cold_pages_batch_tensor(blobs, toks2, "t", "s", "m", 5)
    ko, vo = torch.zeros_like(k), torch.zeros_like(v)
    codec.decode_cold_pages_peak_into(out, toks, ko, vo, "t", "s", "m", 5)

    names = {c[0] for c in rec.calls}
    assert names == {"fused_encode_cold_pages_peak_into_cpu", "fused_encode_cold_pages_batch_cpu",
                     "fused_encode_cold_page_cpu", "fused_decode_cold_page_cpu",
                     "fused_decode_cold_pages_batch_cpu", "fused_decode_cold_pages_peak_into_cpu"}
    for name, args, kwargs in rec.calls:
        sig = inspect.signature(getattr(fused_ext, name))
        sig.bind(*args, **kwargs)  # raises TypeError when the boundary differs
    # the KAT entry points, as the reference module binds them (positional)
    inspect.signature(fused_ext.chacha20_rfc8439_xor_cpu).bind(torch.zeros(4, dtype=torch.uint8),
                                                                torch.zeros(32, dtype=torch.uint8), 1,
                                                                torch.zeros(12, dtype=torch.uint8))
    inspect.signature(fused_ext.siphash24_128_cpu).bind(torch.zeros(4, dtype=torch.uint8), 1, 2)


def test_pybind_argument_names_match(reference):
    """Named arguments of the reference module (its pybind py::arg list) exist on fused_ext."""
    from ztcp_b200 import fused_ext

    mod = reference[0]
    for name in ("fused_encode_cold_page_cpu", "fused_decode_cold_page_cpu", "fused_encode_cold_pages_batch_cpu",
                 "fused_encode_cold_pages_peak_into_cpu", "fused_decode_cold_pages_batch_cpu",
                 "fused_decode_cold_pages_peak_into_cpu"):
        doc = getattr(mod, name).__doc__.splitlines()[0]
        ref_args = [a.split(":")[0].strip() for a in doc[doc.index("(") + 1:doc.index(")")].split(",")]
        ours = list(inspect.signature(getattr(fused_ext, name)).parameters)
        assert ours == ref_args, name
