"""Offload pipeline: cold-page egress to host memory and ingress from it, with the host<->device copies
overlapped with the codec.

The reference's offload path is a wrapper call that returns a CPU blob ready for an RDMA put
(native_fused_codec.py:156, "ready for zero-copy RDMA put"); on a GPU the KV pages live in HBM and the
blobs must cross PCIe.  ``OffloadPipeline`` keeps ``slots`` independent slots, each a CUDA stream with
its own device buffers for one batch; ``egress`` enqueues upload (if the pages are in host memory) ->
encode -> download of the blobs into a caller's pinned buffer, ``ingress`` enqueues upload of blobs ->
verify + decrypt + dequantize -> download of K/V and status, and both return a ``Ticket`` at once.  A
slot is reused only after its previous ticket's work has finished (stream order), so up to ``slots``
batches are in flight and both copy directions stay busy while the SMs run other batches.

Every call goes through ``ztcp_b200.codec`` (the C-ABI); keys and AAD fields are the codec's.  Host
buffers must be pinned (``tensor.pin_memory()``) for the copies to be asynchronous.
"""
from __future__ import annotations

import torch

import ctypes as C

from . import capi, codec


class Ticket:
    """One enqueued batch: ``wait()`` blocks until its results are in host memory (and, for ingress,
    raises the reference's error if a page failed; every output page of the batch is then zero)."""

    def __init__(self, event: torch.cuda.Event, status: torch.Tensor | None = None,
                 any_fail: torch.Tensor | None = None):
        self._event = event
        self._status = status
        self._any_fail = any_fail

    def done(self) -> bool:
        return self._event.query()

    def wait(self) -> None:
        self._event.synchronize()
        if self._any_fail is not None:
            codec.raise_for_status(self._status, self._any_fail)


class _Slot:
    def __init__(self, device: torch.device):
        self.stream = torch.cuda.Stream(device=device)
        self.idle = torch.cuda.Event()
        self.idle.record(self.stream)
        self.buffers: dict[str, torch.Tensor] = {}

    def buffer(self, name: str, shape, dtype, device) -> torch.Tensor:
        t = self.buffers.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
            t = torch.empty(shape, dtype=dtype, device=device)
            self.buffers[name] = t
        return t


class OffloadPipeline:
    def __init__(self, device: torch.device | str = "cuda", slots: int = 8):
        if slots < 1:
            raise ValueError("slots must be >= 1")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("OffloadPipeline runs on a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._slots = [_Slot(self.device) for _ in range(slots)]
        self._next = 0

    def _take(self, after: Ticket | None) -> _Slot:
        s = self._slots[self._next]
        self._next = (self._next + 1) % len(self._slots)
        s.stream.wait_event(s.idle)  # the slot's previous batch has left its buffers
        if after is not None:
            s.stream.wait_event(after._event)
        return s

    def _stage(self, s: _Slot, name: str, t: torch.Tensor | None) -> torch.Tensor | None:
        if t is None or t.device == self.device:
            return t
        d = s.buffer(name, t.shape, t.dtype, self.device)
        d.copy_(t, non_blocking=True)
        return d

    def egress(self, k_pages: torch.Tensor, v_pages: torch.Tensor | None, token_hashes: torch.Tensor,
               out_blobs: torch.Tensor, *, rope_dim: int, preset: int, rope_mode: int, expected_payload_bytes: int,
               tenant_id_hash: int, model_id_hash: int, layer_id: int, head_group_id: int, base_sequence_nonce: int,
               keys: capi.Keys, after: Ticket | None = None) -> Ticket:
        """Encode [B, T, H, D] pages (host or device) into `out_blobs` [B, blob_bytes] (host or device).
        `after`: a ticket whose work must finish first (e.g. the call that filled the inputs)."""
        s = self._take(after)
        with torch.cuda.device(self.device), torch.cuda.stream(s.stream):
            kd = self._stage(s, "k", k_pages)
            vd = self._stage(s, "v", v_pages)
            td = self._stage(s, "tok", token_hashes)
            bd = out_blobs if out_blobs.device == self.device else s.buffer("blobs", out_blobs.shape, torch.uint8,
                                                                             self.device)
            codec.encode_pages(kd, vd, td, bd, rope_dim=rope_dim, preset=preset, rope_mode=rope_mode,
                               expected_payload_bytes=expected_payload_bytes, tenant_id_hash=tenant_id_hash,
                               model_id_hash=model_id_hash, layer_id=layer_id, head_group_id=head_group_id,
                               base_sequence_nonce=base_sequence_nonce, keys=keys)
            if bd is not out_blobs:
                out_blobs.copy_(bd, non_blocking=True)
            done = torch.cuda.Event()
            done.record(s.stream)
            s.idle = done
        return Ticket(done)

    def ingress(self, blobs: torch.Tensor, token_hashes: torch.Tensor, out_k: torch.Tensor,
                out_v: torch.Tensor | None, *, rope_dim: int, is_mla: bool, tenant_id_hash: int, model_id_hash: int,
                layer_id: int, keys: capi.Keys, after: Ticket | None = None) -> Ticket:
        """Verify, decrypt and dequantize `blobs` (host or device) into fp16 `out_k`/`out_v` (host or device).
        `after`: a ticket whose work must finish first (e.g. the egress that wrote `blobs`)."""
        s = self._take(after)
        with torch.cuda.device(self.device), torch.cuda.stream(s.stream):
            bd = self._stage(s, "in_blobs", blobs)
            td = self._stage(s, "in_tok", token_hashes)
            kd = out_k if out_k.device == self.device else s.buffer("out_k", out_k.shape, torch.float16, self.device)
            vd = None if out_v is None else (out_v if out_v.device == self.device else
                                             s.buffer("out_v", out_v.shape, torch.float16, self.device))
            st = s.buffer("status", (blobs.shape[0],), torch.int32, self.device)
            fl = s.buffer("fail", (1,), torch.int32, self.device)
            codec.decode_pages(bd, td, kd, vd, rope_dim=rope_dim, is_mla=is_mla, tenant_id_hash=tenant_id_hash,
                               model_id_hash=model_id_hash, layer_id=layer_id, keys=keys, status=st, any_fail=fl)
            if kd is not out_k:
                out_k.copy_(kd, non_blocking=True)
            if vd is not None and vd is not out_v:
                out_v.copy_(vd, non_blocking=True)
            hs = torch.empty((blobs.shape[0],), dtype=torch.int32, pin_memory=True)  # per ticket: the slot
            hf = torch.empty((1,), dtype=torch.int32, pin_memory=True)                 # may be reused first
            hs.copy_(st, non_blocking=True)
            hf.copy_(fl, non_blocking=True)
            done = torch.cuda.Event()
            done.record(s.stream)
            s.idle = done
        return Ticket(done, hs, hf)

    def synchronize(self) -> None:
        for s in self._slots:
            s.idle.synchronize()


def gather(parts: list[torch.Tensor], device: torch.device | str) -> torch.Tensor:
    """Concatenate uint8 blob tensors that live on several GPUs into one [sum of rows, blob_bytes] tensor
    on `device`, with one peer copy (copy engine, cudaMemcpyPeerAsync) per part on the current stream of
    `device`.  All parts must have the same row width."""
    dev = torch.device(device)
    if dev.type != "cuda" or not parts:
        raise RuntimeError("gather needs CUDA parts and a CUDA destination")
    width = parts[0].shape[1]
    for p in parts:
        if p.device.type != "cuda" or p.dtype != torch.uint8 or p.dim() != 2 or p.shape[1] != width:
            raise RuntimeError("gather parts must be 2-D uint8 CUDA tensors of one row width")
    parts = [p.contiguous() for p in parts]
    out = torch.empty((sum(p.shape[0] for p in parts), width), dtype=torch.uint8, device=dev)
    n = len(parts)
    srcs = (C.c_void_p * n)(*[p.data_ptr() for p in parts])
    devs = (C.c_int32 * n)(*[p.device.index for p in parts])
    sizes = (C.c_int64 * n)(*[p.numel() for p in parts])
    for p in parts:  # the copies start once each part's producer (its own device's current stream) is done
        torch.cuda.current_stream(dev).wait_stream(torch.cuda.current_stream(p.device))
    with torch.cuda.device(dev):
        rc = capi.load().ztcp_gather(C.c_void_p(out.data_ptr()), dev.index, srcs, devs, sizes, n,
                                     C.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    capi.check(rc)
    return out
