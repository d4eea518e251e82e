"""GPU-native batch API over the C-ABI: block tables and per-page metadata.

``encode_pages`` / ``decode_pages`` take CUDA tensors that already live on
one device and enqueue the kernels on the current torch stream without
synchronizing.  They are the building blocks of the reference-compatible
module in ``fused_ext`` and of the benchmark.
"""
from __future__ import annotations

import torch

from . import capi

_U64 = (1 << 64) - 1


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# The current stream's raw handle without building a torch.cuda.Stream object (the lookup torch's own
# kernels use); the public call is the fallback.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _stream_arg(device: torch.device, stream) -> int:
    """Raw handle of `stream` (a torch.cuda.Stream on `device`, a raw handle, or None for the current stream)."""
    if stream is None:
        return _stream_handle(device)
    if isinstance(stream, int):
        return stream
    if stream.device != device:
        raise RuntimeError(f"stream must be on {device}, got {stream.device}")
    return stream.cuda_stream


def _on_device(device: torch.device, fn, *args):
    """Call fn(*args) with `device` current (the C-ABI launches on the current device)."""
    if torch.cuda.current_device() == device.index:
        return fn(*args)
    with torch.cuda.device(device):
        return fn(*args)


class PreparedCall:
    """A codec call checked once, with its C-ABI argument blocks built once: calling it enqueues the same
    kernels on `stream` (a torch.cuda.Stream, a raw handle, or None for the current stream) and returns the
    call's device outputs (None for an egress, (status, any_fail) for a decode or verify).

    The tensors are kept alive by the object and read at every call, so their contents may change between
    calls (new K/V, blobs, token hashes or block-table entries); their shapes, devices and addresses may not.
    A block table's entries are checked on the host when the call is prepared and on the device at every
    call (an entry outside the pool fails that page with PAGE_BAD_BLOCK and touches no memory)."""

    __slots__ = ("_fn", "_args", "_dev", "_keep", "_result")

    def __init__(self, fn, args, dev, keep, result=None):
        self._fn, self._args, self._dev, self._keep, self._result = fn, args, dev, keep, result

    def __call__(self, stream=None):
        rc = _on_device(self._dev, self._fn, *self._args, _stream_arg(self._dev, stream))
        if rc != capi.ZTCP_OK:
            capi.check(rc)
        return self._result


def _require_cuda(name: str, t: torch.Tensor, dtypes, device: torch.device | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if device is not None and t.get_device() != device.index:
        raise RuntimeError(f"{name} must be on {device}, got {t.device}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if t.dtype not in dtypes:
        raise RuntimeError(f"{name} must have dtype in {[str(d) for d in dtypes]}, got {t.dtype}")


def _page_batch(n_pages: int, token_hashes: torch.Tensor, block_table, sequence_nonces, layer_ids,
                base_sequence_nonce: int, tenant: int, model: int, layer_id: int, head_group: int,
                options: int = 0, pool_pages: int = 0) -> capi.PageBatch:
    return capi.PageBatch(n_pages, _ptr(block_table), token_hashes.data_ptr(), _ptr(sequence_nonces), _ptr(layer_ids),
                          int(base_sequence_nonce) & _U64, int(tenant) & 0xFFFFFFFF, int(model) & 0xFFFFFFFF,
                          int(layer_id) & 0xFFFF, int(head_group) & 0xFFFF, options, int(pool_pages))


def _check_meta(dev, n, block_table, sequence_nonces, layer_ids, token_hashes):
    _require_cuda("page_token_hashes", token_hashes, (torch.int64, torch.uint64), dev)
    if token_hashes.dim() != 1 or token_hashes.numel() != n:
        raise RuntimeError("page_token_hashes must be 1D with length equal to batch_size")
    if block_table is not None:
        _require_cuda("block_table", block_table, (torch.int32,), dev)
        if block_table.dim() != 1 or block_table.numel() != n:
            raise RuntimeError("block_table must be 1D int32 with one entry per page")
    if sequence_nonces is not None:
        _require_cuda("sequence_nonces", sequence_nonces, (torch.int64, torch.uint64), dev)
        if sequence_nonces.dim() != 1 or sequence_nonces.numel() != n:
            raise RuntimeError("sequence_nonces must be 1D with one entry per page")
    if layer_ids is not None:
        _require_cuda("layer_ids", layer_ids, (torch.int16, torch.uint16), dev)
        if layer_ids.dim() != 1 or layer_ids.numel() != n:
            raise RuntimeError("layer_ids must be 1D int16 with one entry per page")


def _check_block_table(block_table: torch.Tensor | None, pool_pages: int) -> None:
    # kv_block entries index the pool.  The kernels check every entry against the pool size on the device
    # (a bad page is neither read nor written); this host check turns a bad table into an exception before
    # launch, at the cost of one synchronizing reduction.
    if block_table is not None and block_table.numel() > 0:
        lo, hi = torch.aminmax(block_table)
        if int(lo) < 0 or int(hi) >= pool_pages:
            raise RuntimeError(f"block_table entries must lie in [0, {pool_pages})")


def encode_pages(k_pool: torch.Tensor, v_pool: torch.Tensor | None, token_hashes: torch.Tensor,
                 out_blobs: torch.Tensor, *, stream=None, **kw) -> None:
    """Egress of ``out_blobs.shape[0]`` pages from a KV pool [pool_pages, T, H, D] (fp16 or bf16), enqueued
    on `stream` (default: the current stream); keyword arguments as for ``prepare_encode``."""
    prepare_encode(k_pool, v_pool, token_hashes, out_blobs, **kw)(stream)


def prepare_encode(k_pool: torch.Tensor, v_pool: torch.Tensor | None, token_hashes: torch.Tensor,
                   out_blobs: torch.Tensor, *, rope_dim: int, preset: int, rope_mode: int, expected_payload_bytes: int,
                   tenant_id_hash: int, model_id_hash: int, layer_id: int, head_group_id: int,
                   base_sequence_nonce: int, keys: capi.Keys, block_table: torch.Tensor | None = None,
                   sequence_nonces: torch.Tensor | None = None, layer_ids: torch.Tensor | None = None,
                   check_block_table: bool = True, neon_arith: bool = False) -> PreparedCall:
    """Egress of ``out_blobs.shape[0]`` pages from a KV pool [pool_pages, T, H, D] (fp16 or bf16), checked
    and packed once; the returned call enqueues it.

    Page i reads pool block ``block_table[i]`` (default i) and is written to out_blobs[i].  With
    ``neon_arith`` the groups are quantized with the reference's ARM NEON fp16 arithmetic (the bytes its
    ARM build writes) instead of its scalar x86-64 arithmetic.

    The scalar arguments, ``base_sequence_nonce`` among them, are fixed when the call is prepared.  A
    prepared egress that runs again over new data must therefore take fresh nonces through the
    ``sequence_nonces`` tensor (read at every call): one nonce used twice under one key reuses ChaCha20
    keystream.
    """
    dev = k_pool.device
    _require_cuda("k_pages", k_pool, (torch.float16, torch.bfloat16))
    if k_pool.dim() != 4:
        raise RuntimeError("k_pages must have shape [batch, num_tokens, num_heads, head_dim]")
    if v_pool is not None:
        _require_cuda("v_pages", v_pool, (k_pool.dtype,), dev)
        if v_pool.shape != k_pool.shape:
            raise RuntimeError("v_pages shape must match k_pages shape")
    _require_cuda("out_blobs", out_blobs, (torch.uint8,), dev)
    if out_blobs.dim() != 2:
        raise RuntimeError("out_blobs must have shape [batch, total_blob_bytes]")
    n = out_blobs.shape[0]
    if out_blobs.shape[1] != 32 + expected_payload_bytes + 16:
        raise RuntimeError("out_blobs shape must be [batch_size, total_blob_bytes]")
    if block_table is None and n != k_pool.shape[0]:
        raise RuntimeError("out_blobs batch size must match k_pages batch size")
    _check_meta(dev, n, block_table, sequence_nonces, layer_ids, token_hashes)
    if check_block_table:
        _check_block_table(block_table, k_pool.shape[0])
    _, T, H, D = k_pool.shape
    geom = capi.geometry(T, H, D, rope_dim, v_pool is None)
    batch = _page_batch(n, token_hashes, block_table, sequence_nonces, layer_ids, base_sequence_nonce,
                        tenant_id_hash, model_id_hash, layer_id, head_group_id,
                        capi.OPT_NEON_ARITH if neon_arith else 0, k_pool.shape[0])
    dtype = capi.DTYPE_BF16 if k_pool.dtype == torch.bfloat16 else capi.DTYPE_F16
    args = (k_pool.data_ptr(), _ptr(v_pool), dtype, geom, batch, int(preset), int(rope_mode),
            int(expected_payload_bytes), _copy_keys(keys), out_blobs.data_ptr())
    keep = (k_pool, v_pool, token_hashes, out_blobs, block_table, sequence_nonces, layer_ids)
    return PreparedCall(capi.load().ztcp_encode_pages, args, dev, keep)


def _copy_keys(keys: capi.Keys) -> capi.Keys:
    # a prepared call owns its key block: a caller that zeroizes or reuses its own after preparing changes
    # nothing behind the call's back
    return capi.Keys.from_buffer_copy(keys)


def decode_pages(blobs: torch.Tensor, token_hashes: torch.Tensor, out_k: torch.Tensor,
                 out_v: torch.Tensor | None, *, stream=None, **kw):
    """Ingress of ``blobs.shape[0]`` pages into fp16 pools [pool_pages, T, H, D], enqueued on `stream`
    (default: the current stream); keyword arguments as for ``prepare_decode``.  Returns the device tensors
    (status[n] int32, any_fail[1] int32)."""
    return prepare_decode(blobs, token_hashes, out_k, out_v, **kw)(stream)


def prepare_decode(blobs: torch.Tensor, token_hashes: torch.Tensor, out_k: torch.Tensor,
                   out_v: torch.Tensor | None, *, rope_dim: int, is_mla: bool, tenant_id_hash: int,
                   model_id_hash: int, layer_id: int, keys: capi.Keys, block_table: torch.Tensor | None = None,
                   layer_ids: torch.Tensor | None = None, status: torch.Tensor | None = None,
                   any_fail: torch.Tensor | None = None, check_block_table: bool = True,
                   page_fallback: bool = False) -> PreparedCall:
    """Ingress of ``blobs.shape[0]`` pages into fp16 pools [pool_pages, T, H, D], checked and packed once;
    the returned call enqueues verify + decrypt and returns the device tensors (status[n] int32,
    any_fail[1] int32), the same two at every call.  When any page fails, every output page of the batch is
    zeroed -- or, with ``page_fallback``, only the pages whose status is non-zero (the others are decoded).
    """
    dev = blobs.device
    _require_cuda("cold_blobs", blobs, (torch.uint8,))
    if blobs.dim() != 2:
        raise RuntimeError("cold_blobs must have shape [batch, total_blob_bytes]")
    n, blob_bytes = blobs.shape
    _require_cuda("out_k_pages", out_k, (torch.float16,), dev)
    if out_k.dim() != 4:
        raise RuntimeError("out_k_pages must have shape [batch, num_tokens, num_heads, head_dim]")
    if out_v is not None:
        _require_cuda("out_v_pages", out_v, (torch.float16,), dev)
        if out_v.shape != out_k.shape:
            raise RuntimeError("out_v_pages shape must match out_k_pages shape")
    if block_table is None and n != out_k.shape[0]:
        raise RuntimeError("cold_blobs batch size must match out_k_pages batch size")
    _check_meta(dev, n, block_table, None, layer_ids, token_hashes)
    if check_block_table:
        _check_block_table(block_table, out_k.shape[0])
    if status is None:
        status = torch.empty(n, dtype=torch.int32, device=dev)
    if any_fail is None:
        any_fail = torch.empty(1, dtype=torch.int32, device=dev)
    _, T, H, D = out_k.shape
    geom = capi.geometry(T, H, D, rope_dim, is_mla)
    batch = _page_batch(n, token_hashes, block_table, None, layer_ids, 0, tenant_id_hash, model_id_hash,
                        layer_id, 0, capi.OPT_PAGE_FALLBACK if page_fallback else 0, out_k.shape[0])
    args = (blobs.data_ptr(), int(blob_bytes), geom, batch, _copy_keys(keys), out_k.data_ptr(), _ptr(out_v),
            status.data_ptr(), any_fail.data_ptr())
    keep = (blobs, token_hashes, out_k, out_v, block_table, layer_ids)
    return PreparedCall(capi.load().ztcp_decode_pages, args, dev, keep, (status, any_fail))


def verify_pages(blobs: torch.Tensor, token_hashes: torch.Tensor, *, num_tokens: int, num_heads: int,
                 head_dim: int, rope_dim: int, is_mla: bool, tenant_id_hash: int, model_id_hash: int, layer_id: int,
                 keys: capi.Keys, layer_ids: torch.Tensor | None = None, status: torch.Tensor | None = None,
                 any_fail: torch.Tensor | None = None, stream=None):
    """Integrity check of stored blobs without decrypting, enqueued on `stream` (default: the current
    stream); returns device (status[n], any_fail[1])."""
    dev = blobs.device
    _require_cuda("cold_blobs", blobs, (torch.uint8,))
    if blobs.dim() != 2:
        raise RuntimeError("cold_blobs must have shape [batch, total_blob_bytes]")
    n, blob_bytes = blobs.shape
    _check_meta(dev, n, None, None, layer_ids, token_hashes)
    if status is None:
        status = torch.empty(n, dtype=torch.int32, device=dev)
    if any_fail is None:
        any_fail = torch.empty(1, dtype=torch.int32, device=dev)
    geom = capi.geometry(num_tokens, num_heads, head_dim, rope_dim, is_mla)
    batch = _page_batch(n, token_hashes, None, None, layer_ids, 0, tenant_id_hash, model_id_hash, layer_id, 0)
    rc = _on_device(dev, capi.load().ztcp_verify_pages, blobs.data_ptr(), int(blob_bytes), geom, batch, keys,
                    status.data_ptr(), any_fail.data_ptr(), _stream_arg(dev, stream))
    capi.check(rc)
    return status, any_fail


# Exception texts of the reference's batch and single-page decoders (csrc:2236-2244, :1582-1637).
BATCH_MESSAGES = {
    capi.PAGE_BAD_MAGIC: "KV_INTEGRITY_ERROR: Invalid cold-page header magic, version, or flags",
    capi.PAGE_BAD_FLAGS: "KV_INTEGRITY_ERROR: Invalid cold-page header magic, version, or flags",
    capi.PAGE_TRUNCATED: "KV_INTEGRITY_ERROR: Invalid cold-page header magic, version, or flags",
    capi.PAGE_AAD_MISMATCH: "CROSS_TENANT_CONTAMINATION: Cold-page AAD mismatch",
    capi.PAGE_MAC_FAILED: "KV_INTEGRITY_ERROR: Cold-page MAC verification failed",
    capi.PAGE_BAD_BLOCK: "block_table entry outside the KV pool (page neither read nor written)",
}
SINGLE_MESSAGES = {
    capi.PAGE_BAD_MAGIC: "KV_INTEGRITY_ERROR: Invalid cold-page header magic or version",
    capi.PAGE_AAD_MISMATCH: "CROSS_TENANT_CONTAMINATION: Cold-page AAD mismatch",
    capi.PAGE_MAC_FAILED: "KV_INTEGRITY_ERROR: Cold-page MAC verification failed",
    capi.PAGE_BAD_FLAGS: "KV_INTEGRITY_ERROR: Invalid cold-page header flags (preset or rope_mode)",
    capi.PAGE_TRUNCATED: "KV_INTEGRITY_ERROR: Cold-page payload truncated for header flags",
    capi.PAGE_BAD_BLOCK: "block_table entry outside the KV pool (page neither read nor written)",
}


def raise_for_status(status: torch.Tensor, any_fail: torch.Tensor, single: bool = False) -> None:
    """Synchronize on the decode and raise the reference's error for the first failing page."""
    if int(any_fail.item()) == 0:
        return
    st = status.cpu()
    bad = torch.nonzero(st != 0)
    code = int(st[int(bad[0])]) if bad.numel() else capi.PAGE_MAC_FAILED
    raise RuntimeError((SINGLE_MESSAGES if single else BATCH_MESSAGES)[code])
