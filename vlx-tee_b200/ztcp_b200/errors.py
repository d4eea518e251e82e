"""Exceptions of the ZTCP session layer, with the reference's names and hierarchy
(research/baseline_codec/fused_quant_crypto.py:56-73), so callers' handlers and message-prefix checks
behave the same.  A keyring can instead be given the reference module itself (``errors=``), in which
case it raises the reference's own classes."""
from __future__ import annotations


class KVIntegrityError(RuntimeError):
    """A cold KV page failed MAC authentication (tampering / bit-flip)."""


class CrossTenantContaminationError(KVIntegrityError):
    """A cold KV page's AAD does not match the requesting tenant/model/layer."""


class StalePageReplayError(KVIntegrityError):
    """A cold KV page's sequence_nonce is older than the latest slot version."""


class NonceReuseError(ValueError):
    """An encode call would reuse a final ChaCha20 nonce under the same session key."""


class SessionShreddedError(RuntimeError):
    """The session's ephemeral key was crypto-shredded."""
