"""Offload-path hooks: a compact pinned staging ring for cold blobs and an engine-facing page codec over it
with a per-page recompute fallback.

The reference's design (research/paper/main.tex:171-176) has a serving engine offload KV pages through
SGLang's ``HiCachePageCodec`` or LMCache's ``DirectBatchBufferSerializer`` into ``MooncakeCompactStagingRing``
views, with the page's identity bound into the 32-byte AAD header, and a per-page fallback on the way back:
a page that fails AAD, MAC or freshness verification is not written to hot memory and is marked as a miss
in the engine's hit bitmap, so the engine recomputes that prefix instead of failing the request.  The
reference repository does not contain these hooks; the classes here define them from that description on
top of the session codec (``ztcp_b200.session.ColdPageCodec``: keyring preflight, nonce burn, commit and
freshness around every call):

* ``CompactStagingRing`` -- pinned host memory holding ``slots`` blobs of one size; ``reserve(n)`` hands out
  ``n`` contiguous slots as a ``StagingView`` (wrapping to the start of the ring when its end is too short)
  and ``release(view)`` returns them.  Views may be released in any order; space is reused in ring order.
* ``HiCachePageCodec`` -- ``store`` encodes GPU pages into a view (device encode, then one asynchronous
  copy into the pinned slots; the view's ``ready`` event marks completion), ``load`` decodes a view's blobs
  back into GPU pages and returns the hit bitmap.  A page whose check fails is zeroed and reported False;
  a shredded session makes every page a miss.
"""
from __future__ import annotations

import collections

import torch

from . import errors as _errors
from .cold_page_spec import ColdPageAAD
from .session import ColdPageCodec


class StagingView:
    """``n`` consecutive slots of a ``CompactStagingRing``: ``blobs`` is the [n, blob_bytes] uint8 view."""

    def __init__(self, ring: "CompactStagingRing", start: int, n: int, end: int):
        self.ring = ring
        self.start = start
        self.n = n
        self.end = end  # ring position after this view (start + n, or n when it wrapped to slot 0)
        self.blobs = ring.buffer[start:start + n]
        self.waste = 0  # slots skipped at the ring's end to make this view contiguous
        self.ready: torch.cuda.Event | None = None
        self.token_hashes: torch.Tensor | None = None
        self.released = False


class CompactStagingRing:
    """Fixed-size blob slots in one pinned host buffer, handed out as contiguous views in ring order."""

    def __init__(self, slots: int, blob_bytes: int, pin: bool = True):
        if slots < 1 or blob_bytes < 1:
            raise ValueError("a staging ring needs at least one slot of at least one byte")
        buf = torch.empty((slots, blob_bytes), dtype=torch.uint8)
        self.buffer = buf.pin_memory() if pin else buf
        self.slots = slots
        self.blob_bytes = blob_bytes
        self._head = 0   # next slot to hand out
        self._used = 0   # slots between the oldest live view's start and the head (including wrap waste)
        self._live: collections.deque[StagingView] = collections.deque()

    @property
    def free_slots(self) -> int:
        return self.slots - self._used

    def reserve(self, n: int) -> StagingView:
        """``n`` contiguous slots; raises RuntimeError when the ring cannot hold them now."""
        if n < 1 or n > self.slots:
            raise ValueError(f"a view holds 1..{self.slots} slots, asked for {n}")
        start, waste = self._head, 0
        if start + n > self.slots:  # skip the ring's short tail and wrap to slot 0
            waste = self.slots - start
            start = 0
        if self._used + waste + n > self.slots:
            raise RuntimeError(f"staging ring full: {n} slots asked, {self.free_slots} free")
        self._used += waste + n
        self._head = (start + n) % self.slots
        view = StagingView(self, start, n, start + n)
        view.waste = waste
        self._live.append(view)
        return view

    def release(self, view: StagingView) -> None:
        """Return a view's slots; the space is reused once every older view is released too."""
        if view.ring is not self or view.released:
            raise ValueError("view is not a live view of this ring")
        view.released = True
        while self._live and self._live[0].released:
            v = self._live.popleft()
            self._used -= v.waste + v.n
        if not self._live:
            self._used = 0


class HiCachePageCodec:
    """An engine's page codec: GPU KV pages <-> staging-ring views of encrypted cold blobs."""

    def __init__(self, session_codec: ColdPageCodec, ring: CompactStagingRing):
        self.codec = session_codec
        self.ring = ring
        self.device = session_codec.device

    def store(self, k_pages: torch.Tensor, v_pages: torch.Tensor | None, page_token_hashes_i64: torch.Tensor,
              tenant_id: str, session_id: str, aad_template: ColdPageAAD) -> StagingView:
        """Encode a batch of pages into a new view of the ring (page b gets sequence_nonce base + b).  The
        copy into pinned memory is asynchronous: ``view.ready`` is recorded on the current stream after it."""
        n = page_token_hashes_i64.numel()
        blob = self.codec.geometry.cold_blob_bytes(aad_template.preset, aad_template.rope_mode)
        if blob != self.ring.blob_bytes:
            raise RuntimeError(f"ring slots hold {self.ring.blob_bytes}-byte blobs, this batch needs {blob}")
        view = self.ring.reserve(n)
        try:
            out = torch.empty((n, blob), dtype=torch.uint8, device=self.device)
            self.codec.encode_cold_pages_peak_into(k_pages, v_pages, page_token_hashes_i64, out, tenant_id,
                                                   session_id, aad_template)
            view.blobs.copy_(out, non_blocking=True)
            view.ready = torch.cuda.Event()
            view.ready.record()
            view.token_hashes = page_token_hashes_i64.detach().to("cpu").clone()
        except BaseException:
            self.ring.release(view)
            raise
        return view

    def load(self, view: StagingView, out_k_pages: torch.Tensor, out_v_pages: torch.Tensor | None,
             expected_tenant_id: str, session_id: str, expected_model_id: str, expected_layer_id: int,
             expected_token_hashes_i64: torch.Tensor | None = None,
             min_sequence_nonce: int | None = None) -> torch.Tensor:
        """Decode a view's blobs into GPU pages; returns the hit bitmap (CPU bool [n]).  False pages are zero
        in the outputs and must be recomputed; a shredded session returns all False."""
        if view.released:
            raise ValueError("view was released")
        toks = view.token_hashes if expected_token_hashes_i64 is None else expected_token_hashes_i64
        if view.ready is not None:
            torch.cuda.current_stream(self.device).wait_event(view.ready)
        blobs = view.blobs.to(self.device, non_blocking=True)
        shredded = getattr(self.codec.errors, "SessionShreddedError", _errors.SessionShreddedError)
        try:
            return self.codec.decode_cold_pages_partial(blobs, toks, out_k_pages, out_v_pages, expected_tenant_id,
                                                        session_id, expected_model_id, expected_layer_id,
                                                        min_sequence_nonce)
        except shredded:  # raised before (or while) decoding: no page may reach hot memory
            out_k_pages.zero_()
            if out_v_pages is not None:
                out_v_pages.zero_()
            return torch.zeros(view.n, dtype=torch.bool)
