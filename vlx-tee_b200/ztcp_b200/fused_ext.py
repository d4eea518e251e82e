"""Drop-in replacement for the reference's native codec module.

The reference wrapper ``NativeCppFusedColdPageCodec`` keeps its compiled
module in ``self._ext`` (research/baseline_codec/native_fused_codec.py:78)
and calls eight functions on it (bound at csrc:2540-2683).  This module offers
the same eight functions with the same names, argument order, defaults
(``k2 = k3 = 0``), return values and error texts, running on the B200 codec
through the C-ABI:

    codec._ext = ztcp_b200.fused_ext

Placement.  Tensors may be CUDA tensors (the GPU-resident KV cache: no copy)
or CPU tensors (staged through the current CUDA device with pinned copies and
returned on the CPU, as the reference returns them).  Calls whose outputs are
CUDA tensors are stream-ordered like any torch CUDA op; decode calls
synchronize because they raise on a failed page, as the reference does.
"""
from __future__ import annotations

import torch

from . import capi, codec
from .cold_page_spec import HEADER_BYTES, TAG_BYTES


def _device_of(*tensors) -> torch.device:
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("the ZTCP B200 codec needs a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _to_dev(t: torch.Tensor | None, dev: torch.device) -> torch.Tensor | None:
    if t is None or (t.is_cuda and t.device == dev):
        return t
    if t.is_cuda:
        return t.to(dev)
    src = t if t.is_pinned() else t.pin_memory()
    return src.to(dev, non_blocking=True)


def _hashes(t: torch.Tensor, n: int, dev: torch.device, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or t.dtype != torch.int64 or not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous int64")
    if t.dim() != 1 or t.numel() != n:
        raise RuntimeError(f"{name} must be 1D with length equal to batch_size")
    return _to_dev(t, dev)


def _overlap(a: torch.Tensor | None, b: torch.Tensor | None) -> bool:
    if a is None or b is None or a.numel() == 0 or b.numel() == 0 or a.device != b.device:
        return False
    a0, b0 = a.data_ptr(), b.data_ptr()
    return a0 < b0 + b.numel() * b.element_size() and b0 < a0 + a.numel() * a.element_size()


def _check_kv(name: str, t: torch.Tensor, dims: int) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_contiguous() or t.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(f"{name} must be contiguous float16 or bfloat16 tensor")
    if t.dim() != dims:
        shape = "[batch, num_tokens, num_heads, head_dim]" if dims == 4 else "[num_tokens, num_heads, head_dim]"
        raise RuntimeError(f"{name} must have shape {shape}")


def _geometry_ok(T, H, D, rope_dim, what):
    if not (T > 0 and H > 0 and D >= 16 and D % 16 == 0):
        raise RuntimeError(f"Invalid {what} dimensions")
    if not (0 <= rope_dim <= D and rope_dim % 16 == 0):
        raise RuntimeError("Invalid rope_dim")


def _encode(k_pages, v_pages_opt, page_token_hashes, out_blobs, preset, rope_mode, rope_dim, expected_payload_bytes,
            tenant_id_hash, model_id_hash, layer_id, head_group_id, base_sequence_nonce, keys):
    _check_kv("k_pages", k_pages, 4)
    B, T, H, D = k_pages.shape
    _geometry_ok(T, H, D, rope_dim, "k_pages")
    if B <= 0:
        raise RuntimeError("Invalid k_pages dimensions")
    if v_pages_opt is not None:
        _check_kv("v_pages", v_pages_opt, 4)
        if v_pages_opt.shape != k_pages.shape:
            raise RuntimeError("v_pages shape must match k_pages shape")
    if not 1 <= int(preset) <= 3:
        raise RuntimeError("Invalid preset (must be 1..3)")
    if not 0 <= int(rope_mode) <= 2:
        raise RuntimeError("Invalid rope_mode (must be 0..2)")
    dev = _device_of(k_pages, v_pages_opt, out_blobs)
    k = _to_dev(k_pages, dev)
    v = _to_dev(v_pages_opt, dev) if v_pages_opt is not None else None
    if v is not None and v.dtype != k.dtype:
        v = v.to(k.dtype)
    hashes = _hashes(page_token_hashes, B, dev, "page_token_hashes")
    out_dev = out_blobs if out_blobs.is_cuda and out_blobs.device == dev else torch.empty(
        out_blobs.shape, dtype=torch.uint8, device=dev)
    codec.encode_pages(k, v, hashes, out_dev, rope_dim=int(rope_dim), preset=int(preset), rope_mode=int(rope_mode),
                       expected_payload_bytes=int(expected_payload_bytes), tenant_id_hash=tenant_id_hash,
                       model_id_hash=model_id_hash, layer_id=layer_id, head_group_id=head_group_id,
                       base_sequence_nonce=base_sequence_nonce, keys=keys)
    if out_dev is not out_blobs:
        out_blobs.copy_(out_dev)
    return out_blobs


def fused_encode_cold_pages_peak_into_cpu(k_pages, v_pages_opt, page_token_hashes, out_blobs, preset, rope_mode,
                                          rope_dim, expected_payload_bytes, tenant_id_hash, model_id_hash, layer_id,
                                          head_group_id, base_sequence_nonce, k0, k1, mk0, mk1, k2=0, k3=0):
    """Batch egress into a caller buffer [B, 32 + payload + 16] (csrc:1904-2004)."""
    if not isinstance(out_blobs, torch.Tensor) or out_blobs.dtype != torch.uint8 or not out_blobs.is_contiguous():
        raise RuntimeError("out_blobs must be contiguous uint8 tensor")
    if out_blobs.dim() != 2:
        raise RuntimeError("out_blobs must have shape [batch, total_blob_bytes]")
    if tuple(out_blobs.shape) != (k_pages.shape[0], HEADER_BYTES + int(expected_payload_bytes) + TAG_BYTES):
        raise RuntimeError("out_blobs shape must be [batch_size, total_blob_bytes]")
    if _overlap(out_blobs, k_pages) or _overlap(out_blobs, page_token_hashes) or _overlap(out_blobs, v_pages_opt):
        raise RuntimeError("out_blobs must not alias or overlap input tensors")
    _encode(k_pages, v_pages_opt, page_token_hashes, out_blobs, preset, rope_mode, rope_dim, expected_payload_bytes,
            tenant_id_hash, model_id_hash, layer_id, head_group_id, base_sequence_nonce,
            capi.keys(k0, k1, k2, k3, mk0, mk1))


def fused_encode_cold_pages_batch_cpu(k_pages, v_pages_opt, page_token_hashes, preset, rope_mode, rope_dim,
                                      expected_payload_bytes, tenant_id_hash, model_id_hash, layer_id, head_group_id,
                                      base_sequence_nonce, k0, k1, mk0, mk1, k2=0, k3=0):
    """Batch egress into a new [B, blob] tensor on the input's device (csrc:1775-1902)."""
    _check_kv("k_pages", k_pages, 4)
    out = torch.empty((k_pages.shape[0], HEADER_BYTES + int(expected_payload_bytes) + TAG_BYTES), dtype=torch.uint8,
                      device=k_pages.device)
    return _encode(k_pages, v_pages_opt, page_token_hashes, out, preset, rope_mode, rope_dim, expected_payload_bytes,
                   tenant_id_hash, model_id_hash, layer_id, head_group_id, base_sequence_nonce,
                   capi.keys(k0, k1, k2, k3, mk0, mk1))


def fused_encode_cold_page_cpu(k_page, v_page_opt, preset, rope_mode, rope_dim, expected_payload_bytes,
                               tenant_id_hash, model_id_hash, layer_id, head_group_id, page_token_hash,
                               sequence_nonce, k0, k1, mk0, mk1, k2=0, k3=0):
    """Single-page egress into a new 1-D blob (csrc:1478-1555)."""
    _check_kv("k_page", k_page, 3)
    if v_page_opt is not None:
        _check_kv("v_page", v_page_opt, 3)
        if v_page_opt.shape != k_page.shape:
            raise RuntimeError("v_page shape must match k_page shape")
    hashes = torch.tensor([int(page_token_hash) & ((1 << 64) - 1)], dtype=torch.uint64).view(torch.int64)
    out = fused_encode_cold_pages_batch_cpu(k_page.unsqueeze(0), None if v_page_opt is None else v_page_opt.unsqueeze(0),
                                            hashes, preset, rope_mode, rope_dim, expected_payload_bytes,
                                            tenant_id_hash, model_id_hash, layer_id, head_group_id, sequence_nonce,
                                            k0, k1, mk0, mk1, k2, k3)
    return out[0]


def _decode(cold_blobs, expected_token_hashes, out_k, out_v, rope_dim, is_mla, tenant, model, layer, keys,
            single=False):
    if not isinstance(cold_blobs, torch.Tensor) or cold_blobs.dtype != torch.uint8 or not cold_blobs.is_contiguous():
        raise RuntimeError("cold_blobs must be contiguous uint8")
    if cold_blobs.dim() != 2:
        raise RuntimeError("cold_blobs must have shape [batch, total_blob_bytes]")
    B, blob_bytes = cold_blobs.shape
    if blob_bytes <= HEADER_BYTES + TAG_BYTES:
        raise RuntimeError("cold_blob too small")
    dev = _device_of(out_k, cold_blobs)
    blobs = _to_dev(cold_blobs, dev)
    hashes = _hashes(expected_token_hashes, B, dev, "expected_token_hashes")
    k_dev = out_k if out_k.is_cuda and out_k.device == dev else torch.empty(out_k.shape, dtype=torch.float16, device=dev)
    v_dev = None
    if out_v is not None:
        v_dev = out_v if out_v.is_cuda and out_v.device == dev else torch.empty(out_v.shape, dtype=torch.float16,
                                                                                 device=dev)
    status, any_fail = codec.decode_pages(blobs, hashes, k_dev, v_dev, rope_dim=int(rope_dim), is_mla=bool(is_mla),
                                          tenant_id_hash=tenant, model_id_hash=model, layer_id=layer, keys=keys)
    if k_dev is not out_k:
        out_k.copy_(k_dev)
    if v_dev is not None and v_dev is not out_v:
        out_v.copy_(v_dev)
    codec.raise_for_status(status, any_fail, single=single)


def fused_decode_cold_pages_peak_into_cpu(cold_blobs, expected_token_hashes, out_k_pages, out_v_pages_opt, rope_dim,
                                          is_mla_single_buffer, expected_tenant_hash, expected_model_hash,
                                          expected_layer_id, k0, k1, mk0, mk1, k2=0, k3=0):
    """Batch ingress into caller fp16 buffers; any failing page zeroes every output (csrc:2250-2496)."""
    if not isinstance(out_k_pages, torch.Tensor) or out_k_pages.dtype != torch.float16 or not out_k_pages.is_contiguous():
        raise RuntimeError("out_k_pages must be contiguous float16")
    if out_k_pages.dim() != 4:
        raise RuntimeError("out_k_pages must have shape [batch, num_tokens, num_heads, head_dim]")
    B, T, H, D = out_k_pages.shape
    _geometry_ok(T, H, D, rope_dim, "out_k_pages")
    if cold_blobs.dim() != 2 or cold_blobs.shape[0] != B:
        raise RuntimeError("cold_blobs batch size must match out_k_pages batch size")
    if _overlap(out_k_pages, cold_blobs) or _overlap(out_k_pages, expected_token_hashes):
        raise RuntimeError("out_k_pages must not alias or overlap input tensors")
    if not is_mla_single_buffer:
        if out_v_pages_opt is None:
            raise RuntimeError("out_v_pages is required for non-MLA geometry")
        if out_v_pages_opt.dtype != torch.float16 or not out_v_pages_opt.is_contiguous():
            raise RuntimeError("out_v_pages must be contiguous float16")
        if out_v_pages_opt.shape != out_k_pages.shape:
            raise RuntimeError("out_v_pages shape must match out_k_pages shape")
        if _overlap(out_k_pages, out_v_pages_opt):
            raise RuntimeError("out_k_pages and out_v_pages must not alias or overlap in memory")
        if _overlap(out_v_pages_opt, cold_blobs) or _overlap(out_v_pages_opt, expected_token_hashes):
            raise RuntimeError("out_v_pages must not alias or overlap input tensors")
    out_v = None if is_mla_single_buffer else out_v_pages_opt
    _decode(cold_blobs, expected_token_hashes, out_k_pages, out_v, rope_dim, is_mla_single_buffer,
            expected_tenant_hash, expected_model_hash, expected_layer_id, capi.keys(k0, k1, k2, k3, mk0, mk1))


def fused_decode_cold_pages_batch_cpu(cold_blobs, expected_token_hashes, num_tokens, num_heads, head_dim, rope_dim,
                                      is_mla_single_buffer, expected_tenant_hash, expected_model_hash,
                                      expected_layer_id, k0, k1, mk0, mk1, k2=0, k3=0):
    """Batch ingress into new fp16 tensors on the blobs' device (csrc:2006-2248)."""
    _geometry_ok(num_tokens, num_heads, head_dim, rope_dim, "KV geometry")
    if not isinstance(cold_blobs, torch.Tensor) or cold_blobs.dim() != 2:
        raise RuntimeError("cold_blobs must have shape [batch, total_blob_bytes]")
    B = cold_blobs.shape[0]
    shape = (B, num_tokens, num_heads, head_dim)
    k = torch.empty(shape, dtype=torch.float16, device=cold_blobs.device)
    v = None if is_mla_single_buffer else torch.empty(shape, dtype=torch.float16, device=cold_blobs.device)
    _decode(cold_blobs, expected_token_hashes, k, v, rope_dim, is_mla_single_buffer, expected_tenant_hash,
            expected_model_hash, expected_layer_id, capi.keys(k0, k1, k2, k3, mk0, mk1))
    return k, v


def fused_decode_cold_page_cpu(cold_blob, num_tokens, num_heads, head_dim, rope_dim, is_mla_single_buffer,
                               expected_tenant_hash, expected_model_hash, expected_layer_id, expected_token_hash,
                               k0, k1, mk0, mk1, k2=0, k3=0):
    """Single-blob ingress into new fp16 tensors (csrc:1557-1773); raises the single-page messages."""
    if not isinstance(cold_blob, torch.Tensor) or cold_blob.dtype != torch.uint8 or not cold_blob.is_contiguous():
        raise RuntimeError("cold_blob must be contiguous uint8")
    if cold_blob.dim() != 1:
        raise RuntimeError("cold_blob must be a 1D tensor")
    if cold_blob.numel() <= HEADER_BYTES + TAG_BYTES:
        raise RuntimeError("cold_blob too small")
    _geometry_ok(num_tokens, num_heads, head_dim, rope_dim, "KV geometry")
    shape = (1, num_tokens, num_heads, head_dim)
    k = torch.empty(shape, dtype=torch.float16, device=cold_blob.device)
    v = None if is_mla_single_buffer else torch.empty(shape, dtype=torch.float16, device=cold_blob.device)
    hashes = torch.tensor([int(expected_token_hash) & ((1 << 64) - 1)], dtype=torch.uint64).view(torch.int64)
    _decode(cold_blob.unsqueeze(0), hashes, k, v, rope_dim, is_mla_single_buffer, expected_tenant_hash,
            expected_model_hash, expected_layer_id, capi.keys(k0, k1, k2, k3, mk0, mk1), single=True)
    return k[0], None if v is None else v[0]


def chacha20_rfc8439_xor_cpu(data_u8, key_u8, initial_counter, nonce_u8):
    """RFC 8439 keystream XOR of a uint8 tensor (csrc:2499-2523)."""
    if not isinstance(data_u8, torch.Tensor) or data_u8.dtype != torch.uint8 or not data_u8.is_contiguous():
        raise RuntimeError("data_u8 must be contiguous uint8")
    if key_u8.numel() != 32 or not key_u8.is_contiguous():
        raise RuntimeError("key_u8 must be 32-byte uint8")
    if nonce_u8.numel() != 12 or not nonce_u8.is_contiguous():
        raise RuntimeError("nonce_u8 must be 12-byte uint8")
    dev = _device_of(data_u8)
    src = _to_dev(data_u8, dev)
    dst = torch.empty_like(src)
    key = bytes(key_u8.cpu().numpy().tobytes())
    nonce = bytes(nonce_u8.cpu().numpy().tobytes())
    with torch.cuda.device(dev):
        rc = capi.load().ztcp_chacha20_xor(src.data_ptr() if src.numel() else None, dst.data_ptr() if dst.numel() else None,
                                           src.numel(), key, int(initial_counter) & 0xFFFFFFFF, nonce,
                                           torch.cuda.current_stream(dev).cuda_stream)
    capi.check(rc)
    return dst if data_u8.is_cuda else dst.cpu()


def siphash24_128_cpu(data_u8, mk0, mk1):
    """SipHash-2-4 with 128-bit output of a uint8 tensor (csrc:2525-2538)."""
    if not isinstance(data_u8, torch.Tensor) or data_u8.dtype != torch.uint8 or not data_u8.is_contiguous():
        raise RuntimeError("data_u8 must be contiguous uint8")
    dev = _device_of(data_u8)
    src = _to_dev(data_u8, dev)
    out = torch.empty(16, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        rc = capi.load().ztcp_siphash24_128(src.data_ptr() if src.numel() else None, src.numel(),
                                            int(mk0) & ((1 << 64) - 1), int(mk1) & ((1 << 64) - 1), out.data_ptr(),
                                            torch.cuda.current_stream(dev).cuda_stream)
    capi.check(rc)
    return out if data_u8.is_cuda else out.cpu()
