"""GPU-native session codec: the reference wrapper's interface on CUDA tensors.

``ColdPageCodec`` offers the six public methods of the reference's ``NativeCppFusedColdPageCodec``
(research/baseline_codec/native_fused_codec.py:148-606) with the same argument names and the same
keyring protocol around every call -- egress: preflight (nonces burned) -> begin -> encode -> commit ->
release (:157-215); ingress: begin -> decode (tag, AAD, flags checked on the GPU) -> freshness of the
decoded headers -> finish, outputs zeroed on any failure (:228-282, :372-444) -- but the KV pages, blobs
and outputs may live on the GPU (the reference wrapper reads headers with ``.numpy()`` and so works on CPU
tensors only).  Headers are parsed for the freshness check by the C++ ledger (one 32-byte row per page
crosses to the host), and the keyring's per-page tables are the C++ ledger's when the keyring is a
``ztcp_b200.keyring.SessionKeyRing``.  Any object with the reference keyring's methods also works (for
example the reference's own ``EphemeralSessionKeyRing``).

Tensors on the CPU are staged to the codec's device and results come back on the CPU; CUDA tensors are
used in place.  Egress calls are stream-ordered (the blobs are ready when the current stream reaches
them); ingress calls synchronize, because they must raise before returning pages.
"""
from __future__ import annotations

import struct

import numpy as np
import torch

from . import capi, codec, ledger
from . import errors as _errors
from .cold_page_spec import HEADER_BYTES, ColdPageAAD, ColdPageGeometry, hash32
from .keyring import SessionKeyRing

_M64 = 0xFFFFFFFFFFFFFFFF


def _keys(enc_key: bytes, mac_key: bytes) -> capi.Keys:
    k0, k1, k2, k3 = struct.unpack("<QQQQ", enc_key[:32])
    mk0, mk1 = struct.unpack("<QQ", mac_key[:16])
    return capi.keys(k0, k1, k2, k3, mk0, mk1)


def _overlap(a: torch.Tensor | None, b: torch.Tensor | None) -> bool:
    if a is None or b is None or a.numel() == 0 or b.numel() == 0 or a.device != b.device:
        return False
    a0, b0 = a.data_ptr(), b.data_ptr()
    return a0 < b0 + b.numel() * b.element_size() and b0 < a0 + a.numel() * a.element_size()


class ColdPageCodec:
    def __init__(self, geometry: ColdPageGeometry, keyring, device: torch.device | str | None = None):
        self.geometry = geometry
        self.keyring = keyring
        self.errors = getattr(keyring, "errors", _errors)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type != "cuda":
            raise RuntimeError("ColdPageCodec runs on a CUDA device")

    # ---- helpers -----------------------------------------------------------------------------------
    def _dev(self, t: torch.Tensor | None) -> torch.Tensor | None:
        if t is None or t.device == self.device:
            return t
        return t.contiguous().pin_memory().to(self.device, non_blocking=True)

    def _token_hashes(self, page_token_hashes_i64: torch.Tensor) -> tuple[torch.Tensor, np.ndarray]:
        t = page_token_hashes_i64
        if not isinstance(t, torch.Tensor) or t.dtype not in (torch.int64, torch.uint64) or t.dim() != 1 or t.numel() < 1:
            raise RuntimeError("page_token_hashes_i64 must be a non-empty 1D int64 tensor, got "
                               f"{type(t).__name__ if not isinstance(t, torch.Tensor) else (tuple(t.shape), t.dtype)}")
        host = t.detach().to("cpu").contiguous().numpy().view(np.uint64)
        return self._dev(t.contiguous()), host

    def _check_pages(self, k: torch.Tensor, v: torch.Tensor | None, n: int | None, what: str) -> None:
        g = self.geometry
        exp = (g.num_tokens, g.num_kv_heads, g.head_dim) if n is None else (n, g.num_tokens, g.num_kv_heads, g.head_dim)
        if tuple(k.shape) != exp:
            raise RuntimeError(f"{what} k shape {tuple(k.shape)} does not match geometry {exp}")
        if not g.is_mla_single_buffer and (v is None or tuple(v.shape) != exp):
            raise RuntimeError(f"{what} v shape {None if v is None else tuple(v.shape)} does not match geometry {exp}")

    def _keyring_tokens(self, host: np.ndarray):
        return host if isinstance(self.keyring, SessionKeyRing) else [int(x) for x in host]

    def _map_codec_error(self, exc: RuntimeError):
        msg = str(exc)
        if "CROSS_TENANT_CONTAMINATION" in msg:
            return self.errors.CrossTenantContaminationError(msg)
        if "KV_INTEGRITY_ERROR" in msg:
            return self.errors.KVIntegrityError(msg)
        return None

    # ---- egress ------------------------------------------------------------------------------------
    def _egress(self, k: torch.Tensor, v: torch.Tensor | None, toks: torch.Tensor, out: torch.Tensor,
                tenant_id: str, session_id: str, aad: ColdPageAAD) -> None:
        toks_dev, toks_host = self._token_hashes(toks)
        staged, slots, last = self.keyring.preflight_validate_egress(
            tenant_id=tenant_id, session_id=session_id, model_id_hash=aad.model_id_hash, layer_id=aad.layer_id,
            head_group_id=aad.head_group_id, base_sequence_nonce=aad.sequence_nonce,
            token_hashes=self._keyring_tokens(toks_host))
        try:
            enc_key, mac_key = self.keyring.begin_egress_execution(tenant_id=tenant_id, session_id=session_id,
                                                                   staged_nonces=staged)
            self._check_pages(k, v, toks_host.size, "batch")
            payload = self.geometry.payload_bytes(aad.preset, aad.rope_mode)
            kd, vd = self._dev(k), self._dev(v)
            od = out if out.device == self.device else torch.empty(out.shape, dtype=torch.uint8, device=self.device)
            codec.encode_pages(kd, vd, toks_dev, od, rope_dim=self.geometry.rope_dim, preset=int(aad.preset),
                               rope_mode=int(aad.rope_mode), expected_payload_bytes=payload,
                               tenant_id_hash=aad.tenant_id_hash, model_id_hash=aad.model_id_hash,
                               layer_id=aad.layer_id, head_group_id=aad.head_group_id,
                               base_sequence_nonce=aad.sequence_nonce & _M64, keys=_keys(enc_key, mac_key))
            if od is not out:
                out.copy_(od)
            try:
                self.keyring.commit_egress(tenant_id=tenant_id, session_id=session_id, staged_nonces=staged,
                                           staged_slots=slots, last_seq=last)
            except BaseException:
                out.zero_()
                raise
        finally:
            self.keyring.release_egress_reservation(tenant_id=tenant_id, session_id=session_id, staged_nonces=staged)

    def encode_cold_pages_peak_into(self, k_pages: torch.Tensor, v_pages: torch.Tensor | None,
                                    page_token_hashes_i64: torch.Tensor, out_blobs: torch.Tensor, tenant_id: str,
                                    session_id: str, aad_template: ColdPageAAD) -> None:
        """Batch egress into a caller's [B, blob_bytes] uint8 tensor; page b gets sequence_nonce base + b."""
        blob = self.geometry.cold_blob_bytes(aad_template.preset, aad_template.rope_mode)
        if out_blobs.dtype != torch.uint8 or out_blobs.dim() != 2 or tuple(out_blobs.shape) != (
                page_token_hashes_i64.numel(), blob):
            raise RuntimeError(f"out_blobs must be uint8 [{page_token_hashes_i64.numel()}, {blob}], got "
                               f"{tuple(out_blobs.shape)} {out_blobs.dtype}")
        if _overlap(out_blobs, k_pages) or _overlap(out_blobs, v_pages) or _overlap(out_blobs, page_token_hashes_i64):
            raise RuntimeError("Peak egress output tensor must not alias or overlap input tensors")
        self._egress(k_pages, v_pages, page_token_hashes_i64, out_blobs, tenant_id, session_id, aad_template)

    def encode_cold_pages_batch_tensor(self, k_pages: torch.Tensor, v_pages: torch.Tensor | None,
                                       page_token_hashes_i64: torch.Tensor, tenant_id: str, session_id: str,
                                       aad_template: ColdPageAAD) -> torch.Tensor:
        """Batch egress; returns [B, blob_bytes] uint8 on the device of k_pages."""
        blob = self.geometry.cold_blob_bytes(aad_template.preset, aad_template.rope_mode)
        out = torch.empty((page_token_hashes_i64.numel(), blob), dtype=torch.uint8, device=k_pages.device)
        self._egress(k_pages, v_pages, page_token_hashes_i64, out, tenant_id, session_id, aad_template)
        return out

    def encode_cold_page_tensor(self, k_page: torch.Tensor, v_page: torch.Tensor | None, tenant_id: str,
                                session_id: str, aad: ColdPageAAD) -> torch.Tensor:
        """One page -> 1-D uint8 blob on the device of k_page."""
        self._check_pages(k_page, v_page, None, "page")
        toks = torch.tensor([aad.page_token_hash & _M64], dtype=torch.uint64).view(torch.int64)
        out = torch.empty((1, self.geometry.cold_blob_bytes(aad.preset, aad.rope_mode)), dtype=torch.uint8,
                          device=k_page.device)
        self._egress(k_page.unsqueeze(0), None if v_page is None else v_page.unsqueeze(0), toks, out, tenant_id,
                     session_id, aad)
        return out[0]

    # ---- ingress -----------------------------------------------------------------------------------
    def _ingress(self, blobs: torch.Tensor, toks: torch.Tensor, out_k: torch.Tensor, out_v: torch.Tensor | None,
                 tenant_id: str, session_id: str, model_id: str, layer_id: int, min_sequence_nonce: int | None,
                 expected_sequence_nonce: int | None, single: bool) -> None:
        gen, enc_key, mac_key = self.keyring.begin_ingress(tenant_id, session_id)
        try:
            toks_dev, toks_host = self._token_hashes(toks)
            n = toks_host.size
            if blobs.dim() != 2 or blobs.shape[0] != n or blobs.dtype != torch.uint8:
                raise RuntimeError(f"cold blobs must be uint8 [batch, blob_bytes] with batch={n}, got "
                                   f"{tuple(blobs.shape)} {blobs.dtype}")
            self._check_pages(out_k, out_v, n, "output")
            bd = self._dev(blobs.contiguous())
            kd = out_k if out_k.device == self.device else torch.empty(out_k.shape, dtype=torch.float16,
                                                                         device=self.device)
            vd = None if out_v is None else (out_v if out_v.device == self.device else
                                             torch.empty(out_v.shape, dtype=torch.float16, device=self.device))
            status, fail = codec.decode_pages(bd, toks_dev, kd, vd, rope_dim=self.geometry.rope_dim,
                                              is_mla=bool(self.geometry.is_mla_single_buffer),
                                              tenant_id_hash=hash32(tenant_id), model_id_hash=hash32(model_id),
                                              layer_id=layer_id, keys=_keys(enc_key, mac_key))
            try:
                codec.raise_for_status(status, fail, single=single)
            except RuntimeError as exc:
                mapped = self._map_codec_error(exc)
                if mapped is None:
                    raise
                raise mapped from exc
            records = ledger.records_from_headers(bd[:, :HEADER_BYTES].cpu().numpy())
            if single:
                r = records[0]
                self.keyring.verify_and_update_freshness(
                    tenant_id=tenant_id, session_id=session_id, model_id_hash=int(r["model_id_hash"]),
                    layer_id=int(r["layer_id"]), head_group_id=int(r["head_group_id"]),
                    page_token_hash=int(r["page_token_hash"]), sequence_nonce=int(r["sequence_nonce"]),
                    min_sequence_nonce=min_sequence_nonce, expected_sequence_nonce=expected_sequence_nonce,
                    expected_generation=gen)
            else:
                recs = records if isinstance(self.keyring, SessionKeyRing) else [tuple(int(x) for x in r)
                                                                                 for r in records]
                self.keyring.verify_and_update_freshness_batch(tenant_id=tenant_id, session_id=session_id,
                                                               records=recs, min_sequence_nonce=min_sequence_nonce,
                                                               expected_generation=gen)
            self.keyring.finish_ingress(tenant_id, session_id, gen)
            if kd is not out_k:
                out_k.copy_(kd)
            if vd is not None and vd is not out_v:
                out_v.copy_(vd)
        except BaseException:
            out_k.zero_()
            if out_v is not None:
                out_v.zero_()
            raise

    def decode_cold_pages_partial(self, cold_blobs_u8: torch.Tensor, expected_token_hashes_i64: torch.Tensor,
                                  out_k_pages: torch.Tensor, out_v_pages: torch.Tensor | None,
                                  expected_tenant_id: str, session_id: str, expected_model_id: str,
                                  expected_layer_id: int, min_sequence_nonce: int | None = None) -> torch.Tensor:
        """Batch ingress with a per-page fallback: returns a CPU bool tensor, True for each page decoded into
        the outputs, False for each page that failed its header, AAD, MAC, flags or freshness check (its
        outputs are zeroed and its slot watermark is left as it was).  A session-level failure (the key
        shredded before or during the call) still raises, with every output zeroed.  This is the per-page
        recovery the reference's design describes for an engine's offload hook (paper main.tex:174); the
        reference's own decoders are all-or-nothing (``decode_cold_pages_peak_into``)."""
        if (_overlap(out_k_pages, out_v_pages) or _overlap(out_k_pages, cold_blobs_u8)
                or _overlap(out_v_pages, cold_blobs_u8)):
            raise RuntimeError("Peak ingress output tensors must not alias or overlap each other or input tensors")
        tenant_id = expected_tenant_id
        gen, enc_key, mac_key = self.keyring.begin_ingress(tenant_id, session_id)
        out_k, out_v = out_k_pages, out_v_pages
        try:
            toks_dev, toks_host = self._token_hashes(expected_token_hashes_i64)
            n = toks_host.size
            if cold_blobs_u8.dim() != 2 or cold_blobs_u8.shape[0] != n or cold_blobs_u8.dtype != torch.uint8:
                raise RuntimeError(f"cold blobs must be uint8 [batch, blob_bytes] with batch={n}, got "
                                   f"{tuple(cold_blobs_u8.shape)} {cold_blobs_u8.dtype}")
            self._check_pages(out_k, out_v, n, "output")
            bd = self._dev(cold_blobs_u8.contiguous())
            kd = out_k if out_k.device == self.device else torch.empty(out_k.shape, dtype=torch.float16,
                                                                         device=self.device)
            vd = None if out_v is None else (out_v if out_v.device == self.device else
                                             torch.empty(out_v.shape, dtype=torch.float16, device=self.device))
            status, _ = codec.decode_pages(bd, toks_dev, kd, vd, rope_dim=self.geometry.rope_dim,
                                           is_mla=bool(self.geometry.is_mla_single_buffer),
                                           tenant_id_hash=hash32(tenant_id), model_id_hash=hash32(expected_model_id),
                                           layer_id=expected_layer_id, keys=_keys(enc_key, mac_key),
                                           page_fallback=True)
            hits = (status == 0).cpu()
            records = ledger.records_from_headers(bd[:, :HEADER_BYTES].cpu().numpy())
            for i in np.flatnonzero(hits.numpy()):
                r = records[i]
                try:
                    self.keyring.verify_and_update_freshness(
                        tenant_id=tenant_id, session_id=session_id, model_id_hash=int(r["model_id_hash"]),
                        layer_id=int(r["layer_id"]), head_group_id=int(r["head_group_id"]),
                        page_token_hash=int(r["page_token_hash"]), sequence_nonce=int(r["sequence_nonce"]),
                        min_sequence_nonce=min_sequence_nonce, expected_generation=gen)
                except self.errors.StalePageReplayError:
                    hits[i] = False
            misses = torch.nonzero(~hits).flatten().to(self.device)
            if misses.numel():
                kd.index_fill_(0, misses, 0)
                if vd is not None:
                    vd.index_fill_(0, misses, 0)
            self.keyring.finish_ingress(tenant_id, session_id, gen)
            if kd is not out_k:
                out_k.copy_(kd)
            if vd is not None and vd is not out_v:
                out_v.copy_(vd)
            return hits
        except BaseException:
            out_k.zero_()
            if out_v is not None:
                out_v.zero_()
            raise

    def decode_cold_pages_peak_into(self, cold_blobs_u8: torch.Tensor, expected_token_hashes_i64: torch.Tensor,
                                    out_k_pages: torch.Tensor, out_v_pages: torch.Tensor | None,
                                    expected_tenant_id: str, session_id: str, expected_model_id: str,
                                    expected_layer_id: int, min_sequence_nonce: int | None = None) -> None:
        """Batch ingress into caller-allocated fp16 [B, T, H, D] tensors; all of them zeroed on any failure."""
        if (_overlap(out_k_pages, out_v_pages) or _overlap(out_k_pages, cold_blobs_u8)
                or _overlap(out_v_pages, cold_blobs_u8) or _overlap(out_k_pages, expected_token_hashes_i64)
                or _overlap(out_v_pages, expected_token_hashes_i64)):
            raise RuntimeError("Peak ingress output tensors must not alias or overlap each other or input tensors")
        self._ingress(cold_blobs_u8, expected_token_hashes_i64, out_k_pages, out_v_pages, expected_tenant_id,
                      session_id, expected_model_id, expected_layer_id, min_sequence_nonce, None, single=False)

    def decode_cold_pages_batch_tensor(self, cold_blobs_u8: torch.Tensor, expected_token_hashes_i64: torch.Tensor,
                                       expected_tenant_id: str, session_id: str, expected_model_id: str,
                                       expected_layer_id: int, min_sequence_nonce: int | None = None):
        """Batch ingress; returns (K, V or None) fp16 [B, T, H, D] on the device of the blobs."""
        g = self.geometry
        shape = (expected_token_hashes_i64.numel(), g.num_tokens, g.num_kv_heads, g.head_dim)
        k = torch.empty(shape, dtype=torch.float16, device=cold_blobs_u8.device)
        v = None if g.is_mla_single_buffer else torch.empty_like(k)
        self._ingress(cold_blobs_u8, expected_token_hashes_i64, k, v, expected_tenant_id, session_id,
                      expected_model_id, expected_layer_id, min_sequence_nonce, None, single=False)
        return k, v

    def decode_cold_page_tensor(self, cold_blob_u8: torch.Tensor, expected_tenant_id: str, session_id: str,
                                expected_model_id: str, expected_layer_id: int, expected_token_hash: int,
                                min_sequence_nonce: int | None = None, expected_sequence_nonce: int | None = None):
        """One blob -> (K, V or None) fp16 [T, H, D]; the single-page checks and messages of the reference."""
        g = self.geometry
        shape = (1, g.num_tokens, g.num_kv_heads, g.head_dim)
        k = torch.empty(shape, dtype=torch.float16, device=cold_blob_u8.device)
        v = None if g.is_mla_single_buffer else torch.empty_like(k)
        toks = torch.tensor([expected_token_hash & _M64], dtype=torch.uint64).view(torch.int64)
        self._ingress(cold_blob_u8.reshape(1, -1), toks, k, v, expected_tenant_id, session_id, expected_model_id,
                      expected_layer_id, min_sequence_nonce, expected_sequence_nonce, single=True)
        return k[0], None if v is None else v[0]
