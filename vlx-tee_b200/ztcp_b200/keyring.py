"""Session keyring with the reference's interface and semantics, its per-page tables in C++.

``SessionKeyRing`` is a drop-in for the reference's ``EphemeralSessionKeyRing``
(research/baseline_codec/fused_quant_crypto.py:99-659): the same public methods and argument names, the
same key derivation (HMAC-SHA256 over the deployment pepper, ``tenant:session:gen=N:`` and a fresh
256-bit secret; enc and mac keys under the labels ``ztcp-cold-page-enc-v1\\x01`` /
``ztcp-cold-page-mac-v1\\x02``), the same generation and crypto-shred rules, and the same exceptions and
messages.  What differs is where the per-page work runs: the burned-nonce set, the slot freshness
watermarks and the session's largest sequence nonce live in the C++ ledger (include/ztcp_ledger.h), which
checks a whole batch at once.  The reference walks them page by page in Python (preflight :263-342,
freshness :543-603), which at GPU codec speed costs more than the codec.

Reservations returned by ``preflight_validate_egress`` are opaque objects to pass back to
``begin_egress_execution`` / ``commit_egress`` / ``release_egress_reservation``, as the reference's
wrapper (native_fused_codec.py:157-215) does.
"""
from __future__ import annotations

import hashlib
import hmac
import os
import struct
import threading

import numpy as np

from . import errors as _errors
from . import ledger as _ledger

_M64 = 0xFFFFFFFFFFFFFFFF


class Reservation:
    """Nonces reserved (burned) by one preflight, bound to a key generation, with key snapshots."""

    def __init__(self, handle: _ledger.Reservation, generation: int, ledger_id: int, enc: bytearray, mac: bytearray,
                 first_nonce: bytes):
        self.handle = handle
        self.generation = generation
        self.ledger_id = ledger_id
        self.enc_buf = enc
        self.mac_buf = mac
        self.first_nonce = first_nonce
        self.revoked = False

    def zeroize(self) -> None:
        self.enc_buf[:] = b"\x00" * len(self.enc_buf)
        self.mac_buf[:] = b"\x00" * len(self.mac_buf)

    def __len__(self) -> int:
        return self.handle.pages if self.handle._h else 0


class StagedSlots:
    """The slot watermarks a preflight staged (kept by the ledger reservation); pass back to commit_egress."""

    def __init__(self, reservation: Reservation):
        self.reservation = reservation


class SessionKeyRing:
    """Per-(tenant, session) ephemeral keys, nonce uniqueness, freshness and crypto-shredding."""

    def __init__(self, deployment_pepper: bytes, errors=None):
        if len(deployment_pepper) < 32:
            raise ValueError("deployment_pepper must be at least 32 bytes")
        self.deployment_pepper = deployment_pepper
        self.errors = errors if errors is not None else _errors
        self._lock = threading.RLock()
        self._ledger = _ledger.Ledger()
        self._ledger_ids: dict[tuple[str, str], int] = {}
        self._next_ledger_id = 1
        self._active_keys: dict[tuple[str, str], tuple[bytearray, bytearray, int, int]] = {}
        self._session_generations: dict[tuple[str, str], int] = {}
        self._shredded_generations: dict[tuple[str, str], int] = {}
        self._inflight: dict[tuple[tuple[str, str], int], list[Reservation]] = {}

    # ---- helpers -----------------------------------------------------------------------------------
    @staticmethod
    def pack_chacha20_nonce(sequence_nonce: int, layer_id: int, head_group_id: int) -> bytes:
        """96-bit ChaCha20 nonce: sequence_nonce (64 bits LE) || layer_id << 16 | head_group_id (32 bits LE)."""
        seq = sequence_nonce & _M64
        return struct.pack("<3I", seq & 0xFFFFFFFF, seq >> 32, ((layer_id & 0xFFFF) << 16) | (head_group_id & 0xFFFF))

    def _shredded(self, msg: str):
        return self.errors.SessionShreddedError(msg)

    def _ensure_active_generation_locked(self, cache_key: tuple[str, str]) -> int:
        entry = self._active_keys.get(cache_key)
        if entry is None:
            raise self._shredded(f"Session {cache_key} key is missing or crypto-shredded")
        enc, mac = entry[0], entry[1]
        if len(enc) != 32 or len(mac) != 32 or not any(enc) or not any(mac):
            raise self._shredded(f"Session {cache_key} key buffer was zeroized or crypto-shredded")
        if cache_key not in self._session_generations:
            self._session_generations[cache_key] = self._shredded_generations.get(cache_key, 0) + 1
        return self._session_generations[cache_key]

    def _generation_live(self, cache_key, generation: int) -> bool:
        return (cache_key in self._active_keys and self._session_generations.get(cache_key) == generation
                and self._shredded_generations.get(cache_key, 0) < generation)

    # ---- keys and nonces ---------------------------------------------------------------------------
    def derive_or_get(self, tenant_id: str, session_id: str) -> tuple[bytearray, bytearray, int, int]:
        """Returns (enc_key_32b, mac_key_32b, k0_u64, k1_u64) for the session."""
        with self._lock:
            cache_key = (tenant_id, session_id)
            if cache_key in self._active_keys:
                self._ensure_active_generation_locked(cache_key)
                return self._active_keys[cache_key]
            gen = max(self._session_generations.get(cache_key, 0), self._shredded_generations.get(cache_key, 0)) + 1
            self._session_generations[cache_key] = gen
            secret = bytearray(os.urandom(32))
            try:
                prk = hmac.new(self.deployment_pepper,
                               f"{tenant_id}:{session_id}:gen={gen}:".encode("utf-8") + bytes(secret),
                               hashlib.sha256).digest()
            finally:
                secret[:] = b"\x00" * len(secret)
            enc = bytearray(hmac.new(prk, b"ztcp-cold-page-enc-v1\x01", hashlib.sha256).digest())
            mac = bytearray(hmac.new(prk, b"ztcp-cold-page-mac-v1\x02", hashlib.sha256).digest())
            lid = self._next_ledger_id
            self._next_ledger_id += 1
            self._ledger.open(lid)
            self._ledger_ids[cache_key] = lid
            self._inflight[(cache_key, gen)] = []
            k0, k1 = struct.unpack("<QQ", enc[:16])
            entry = (enc, mac, k0, k1)
            self._active_keys[cache_key] = entry
            return entry

    def next_sequence_nonce(self, tenant_id: str, session_id: str, count: int = 1) -> int:
        """Allocates a fresh monotonic sequence_nonce range [base, base + count) for the session."""
        if count < 1:
            raise ValueError("count must be >= 1")
        with self._lock:
            cache_key = (tenant_id, session_id)
            if cache_key not in self._active_keys:
                self.derive_or_get(tenant_id, session_id)
            self._ensure_active_generation_locked(cache_key)
            return self._ledger.next_nonce(self._ledger_ids[cache_key], count)

    # ---- egress ------------------------------------------------------------------------------------
    def preflight_validate_egress(self, tenant_id: str, session_id: str, model_id_hash: int, layer_id: int,
                                  head_group_id: int, base_sequence_nonce: int, token_hashes):
        """Checks every page for staleness and nonce reuse, then burns the batch's nonces (all or none).

        Returns (reservation, staged_slots, last_seq).  `token_hashes` is a list of ints or a uint64/int64
        array."""
        if token_hashes is None or len(token_hashes) == 0:
            raise ValueError("token_hashes must be non-empty")
        with self._lock:
            cache_key = (tenant_id, session_id)
            if cache_key not in self._active_keys:
                self.derive_or_get(tenant_id, session_id)
            gen = self._ensure_active_generation_locked(cache_key)
            enc, mac = self._active_keys[cache_key][0], self._active_keys[cache_key][1]
            lid = self._ledger_ids[cache_key]
            l_id, g_id = layer_id & 0xFFFF, head_group_id & 0xFFFF
            base = base_sequence_nonce & _M64
            toks = token_hashes
            if isinstance(toks, np.ndarray):
                toks = toks.astype(np.uint64, copy=False)
            try:
                handle = self._ledger.preflight(lid, model_id_hash & 0xFFFFFFFF, l_id, g_id, base, toks)
            except _ledger.LedgerError as e:
                if e.code == _ledger.ESTALE:
                    raise self.errors.StalePageReplayError(
                        f"STALE_PAGE_REPLAY: Cannot encode cold page with stale sequence_nonce={e.err.seq} "
                        f"< latest={e.err.ref}") from None
                nonce = int(e.err.seq).to_bytes(8, "little") + struct.pack("<I", int(e.err.loc))
                raise self.errors.NonceReuseError(
                    f"NONCE_REUSE_DETECTED: Final 96-bit ChaCha20 nonce {nonce.hex()} already used under "
                    f"session {cache_key}") from None
            first = base.to_bytes(8, "little") + struct.pack("<I", (l_id << 16) | g_id)
            res = Reservation(handle, gen, lid, bytearray(enc), bytearray(mac), first)
            self._inflight.setdefault((cache_key, gen), []).append(res)
            return res, StagedSlots(res), handle.last_seq

    def _resolve(self, staged_nonces) -> tuple[int, bool]:
        if isinstance(staged_nonces, Reservation):
            return staged_nonces.generation, staged_nonces.revoked
        return -1, True

    def begin_egress_execution(self, tenant_id: str, session_id: str, staged_nonces) -> tuple[bytes, bytes]:
        """Verifies the reservation's generation is still active; returns immutable key snapshots."""
        with self._lock:
            cache_key = (tenant_id, session_id)
            gen, revoked = self._resolve(staged_nonces)
            if revoked or not self._generation_live(cache_key, gen):
                if isinstance(staged_nonces, Reservation):
                    staged_nonces.zeroize()
                raise self._shredded(f"Session ({tenant_id}, {session_id}) generation {gen} was crypto-shredded "
                                     f"before or during egress")
            r = staged_nonces
            if len(r.enc_buf) != 32 or len(r.mac_buf) != 32 or not any(r.enc_buf) or not any(r.mac_buf):
                r.zeroize()
                raise self._shredded(f"Session ({tenant_id}, {session_id}) generation {gen} key buffer was zeroized")
            return bytes(r.enc_buf), bytes(r.mac_buf)

    def commit_egress(self, tenant_id: str, session_id: str, staged_nonces, staged_slots, last_seq: int) -> None:
        """Raises the staged slot watermarks (never lowers them) once the generation is known to be live."""
        with self._lock:
            cache_key = (tenant_id, session_id)
            gen, revoked = self._resolve(staged_nonces)
            if revoked or not self._generation_live(cache_key, gen):
                if isinstance(staged_nonces, Reservation):
                    staged_nonces.zeroize()
                raise self._shredded(f"Session ({tenant_id}, {session_id}) generation {gen} was crypto-shredded "
                                     f"before commit")
            r = staged_slots.reservation if isinstance(staged_slots, StagedSlots) else staged_nonces
            self._ledger.commit(self._ledger_ids[cache_key], r.handle)

    def release_egress_reservation(self, tenant_id: str, session_id: str, staged_nonces) -> None:
        """Zeroizes the operation's key snapshots and unregisters the reservation."""
        with self._lock:
            if isinstance(staged_nonces, Reservation):
                staged_nonces.zeroize()
                lst = self._inflight.get(((tenant_id, session_id), staged_nonces.generation))
                if lst is not None and staged_nonces in lst:
                    lst.remove(staged_nonces)
                staged_nonces.handle.free()

    # ---- ingress -----------------------------------------------------------------------------------
    def begin_ingress(self, tenant_id: str, session_id: str) -> tuple[int, bytes, bytes]:
        """Captures the active generation and immutable key snapshots for an ingress decode."""
        with self._lock:
            cache_key = (tenant_id, session_id)
            if cache_key not in self._active_keys:
                raise self._shredded(f"Session ({tenant_id}, {session_id}) key is missing or crypto-shredded")
            gen = self._ensure_active_generation_locked(cache_key)
            enc, mac = self._active_keys[cache_key][0], self._active_keys[cache_key][1]
            return gen, bytes(enc), bytes(mac)

    def _check_ingress_generation(self, tenant_id, session_id, expected_generation) -> int:
        cache_key = (tenant_id, session_id)
        if cache_key not in self._active_keys:
            raise self._shredded(f"Session ({tenant_id}, {session_id}) key is missing or crypto-shredded")
        cur = self._ensure_active_generation_locked(cache_key)
        if expected_generation is not None and (
                cur != expected_generation or self._shredded_generations.get(cache_key, 0) >= expected_generation):
            raise self._shredded(f"Session ({tenant_id}, {session_id}) generation {expected_generation} was "
                                 f"crypto-shredded during ingress")
        return self._ledger_ids[cache_key]

    def _stale(self, e: _ledger.LedgerError):
        if e.code == _ledger.EMISMATCH:
            return self.errors.StalePageReplayError(
                f"STALE_PAGE_REPLAY: Cold-page sequence_nonce={e.err.seq} != expected_sequence_nonce={e.err.ref}")
        if e.err.kind == 1:
            return self.errors.StalePageReplayError(
                f"STALE_PAGE_REPLAY: Cold-page sequence_nonce={e.err.seq} < min_sequence_nonce={e.err.ref}")
        return self.errors.StalePageReplayError(
            f"STALE_PAGE_REPLAY: Cold-page sequence_nonce={e.err.seq} is older than latest slot version={e.err.ref}")

    def verify_and_update_freshness(self, tenant_id: str, session_id: str, model_id_hash: int, layer_id: int,
                                    head_group_id: int, page_token_hash: int, sequence_nonce: int,
                                    min_sequence_nonce: int | None = None, expected_sequence_nonce: int | None = None,
                                    expected_generation: int | None = None) -> None:
        """Freshness of one authenticated page: expected nonce, minimum, then the slot watermark."""
        with self._lock:
            lid = self._check_ingress_generation(tenant_id, session_id, expected_generation)
            rec = _ledger.FreshRecord(model_id_hash & 0xFFFFFFFF, layer_id & 0xFFFF, head_group_id & 0xFFFF,
                                      page_token_hash & _M64, sequence_nonce & _M64)
            try:
                self._ledger.freshness_one(lid, rec, None if min_sequence_nonce is None else min_sequence_nonce & _M64,
                                           None if expected_sequence_nonce is None else expected_sequence_nonce & _M64)
            except _ledger.LedgerError as e:
                raise self._stale(e) from None

    def verify_and_update_freshness_batch(self, tenant_id: str, session_id: str, records,
                                          min_sequence_nonce: int | None = None,
                                          expected_generation: int | None = None) -> None:
        """Freshness of a batch of decoded headers, all or nothing.  `records` is a list of
        (model_id_hash, layer_id, head_group_id, page_token_hash, sequence_nonce) tuples or a record array
        (ledger.RECORD_DTYPE, e.g. from ledger.records_from_headers)."""
        with self._lock:
            lid = self._check_ingress_generation(tenant_id, session_id, expected_generation)
            rec = records if isinstance(records, np.ndarray) else _ledger.records_from_tuples(records)
            try:
                self._ledger.freshness_batch(lid, rec, None if min_sequence_nonce is None else min_sequence_nonce & _M64)
            except _ledger.LedgerError as e:
                raise self._stale(e) from None

    def finish_ingress(self, tenant_id: str, session_id: str, expected_generation: int) -> None:
        """Verifies the generation is still active right before decoded tensors are returned."""
        with self._lock:
            if not self._generation_live((tenant_id, session_id), expected_generation):
                raise self._shredded(f"Session ({tenant_id}, {session_id}) generation {expected_generation} was "
                                     f"crypto-shredded during ingress")

    # ---- crypto-shredding --------------------------------------------------------------------------
    def _zeroize_and_remove_session(self, cache_key: tuple[str, str]) -> bool:
        with self._lock:
            gen = self._session_generations.get(cache_key, 1)
            entry = self._active_keys.pop(cache_key, None)
            existed = entry is not None
            if entry is not None:
                entry[0][:] = b"\x00" * len(entry[0])
                entry[1][:] = b"\x00" * len(entry[1])
            for res in self._inflight.pop((cache_key, gen), []):
                res.revoked = True
                res.zeroize()
            lid = self._ledger_ids.pop(cache_key, None)
            if lid is not None:
                self._ledger.close(lid)
            if existed:
                self._shredded_generations[cache_key] = max(self._shredded_generations.get(cache_key, 0), gen)
            return existed

    def crypto_shred_session(self, tenant_id: str, session_id: str) -> bool:
        """Zeroes the session's key buffers, revokes in-flight operations and drops its tables."""
        with self._lock:
            return self._zeroize_and_remove_session((tenant_id, session_id))

    def crypto_shred_tenant(self, tenant_id: str) -> int:
        """Shreds every active session of a tenant; returns how many."""
        with self._lock:
            keys = [k for k in self._active_keys if k[0] == tenant_id]
            for k in keys:
                self._zeroize_and_remove_session(k)
            return len(keys)
