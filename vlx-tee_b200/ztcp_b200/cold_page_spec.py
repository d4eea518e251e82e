"""Cold-page wire format: header, presets, geometry and payload sizes.

Host-side mirror of the reference spec module
(research/baseline_codec/cold_page_spec.py): the same names, enum values,
header struct and size rules, so code written against the reference spec runs
unchanged.  Payload sizes come from the same rule the CUDA library applies
(``ztcp_layout.h``); ``ColdPageGeometry.payload_bytes`` is checked against
``ztcp_spec_payload_bytes`` in the tests.
"""
from __future__ import annotations

import enum
import hashlib
import struct
from dataclasses import dataclass

MAGIC_ZTCP = 0x5A54          # "ZT" little-endian, cold_page_spec.py:47
CODEC_VERSION = 1
HEADER_BYTES = 32
TAG_BYTES = 16
HEADER_STRUCT = struct.Struct("<HBBIIHHQQ")   # cold_page_spec.py:51
GROUP_SIZE = 16


class QuantPreset(enum.IntEnum):
    """cold_page_spec.py:54-59."""

    INT4_SYM = 1    # K and V: symmetric INT4, fp16 scale per 16-group
    K8V4_ASYM = 2   # K: symmetric INT8, V: symmetric INT4 ("asymmetric" bit allocation)
    FP8_ONLY = 3    # K and V: symmetric INT8 (named FP8 in the reference; the codec is INT8)


class RoPEMode(enum.IntEnum):
    """cold_page_spec.py:62-67."""

    QUANTIZE_ALL = 0   # RoPE columns quantized with the rest of K
    PRESERVE_FP8 = 1   # RoPE columns kept in 8 bits (symmetric INT8 + fp16 scales)
    PRESERVE_RAW = 2   # RoPE columns kept as raw fp16


def hash32(text: str) -> int:
    """32-bit domain hash: blake2s digest_size=4, little-endian (cold_page_spec.py:70-73)."""
    return int.from_bytes(hashlib.blake2s(text.encode("utf-8"), digest_size=4).digest(), "little")


def hash64_tokens(token_ids) -> int:
    """64-bit prefix hash of int32 token ids: blake2s digest_size=8 (cold_page_spec.py:76-80)."""
    raw = struct.pack(f"<{len(token_ids)}i", *token_ids)
    return int.from_bytes(hashlib.blake2s(raw, digest_size=8).digest(), "little")


@dataclass(frozen=True)
class ColdPageAAD:
    """Associated data bound into every tag (cold_page_spec.py:83-161)."""

    tenant_id_hash: int
    model_id_hash: int
    layer_id: int
    page_token_hash: int
    sequence_nonce: int
    preset: QuantPreset = QuantPreset.K8V4_ASYM
    rope_mode: RoPEMode = RoPEMode.PRESERVE_FP8
    head_group_id: int = 0

    @classmethod
    def from_context(cls, tenant_id: str, model_id: str, layer_id: int, token_ids, sequence_nonce: int,
                     preset: QuantPreset = QuantPreset.K8V4_ASYM,
                     rope_mode: RoPEMode = RoPEMode.PRESERVE_FP8) -> "ColdPageAAD":
        return cls(hash32(tenant_id), hash32(model_id), layer_id, hash64_tokens(token_ids), sequence_nonce,
                   preset, rope_mode)

    @property
    def flags(self) -> int:
        return (int(self.preset) & 0x0F) | ((int(self.rope_mode) & 0x0F) << 4)

    def pack_header(self) -> bytes:
        return HEADER_STRUCT.pack(
            MAGIC_ZTCP, CODEC_VERSION, self.flags,
            self.tenant_id_hash & 0xFFFFFFFF, self.model_id_hash & 0xFFFFFFFF,
            self.layer_id & 0xFFFF, self.head_group_id & 0xFFFF,
            self.page_token_hash & 0xFFFFFFFFFFFFFFFF, self.sequence_nonce & 0xFFFFFFFFFFFFFFFF,
        )

    @classmethod
    def unpack_header(cls, header_bytes: bytes) -> "ColdPageAAD":
        if len(header_bytes) < HEADER_BYTES:
            raise ValueError(f"Header too short: {len(header_bytes)} < {HEADER_BYTES}")
        magic, version, flags, tenant, model, layer, head_group, tok, seq = HEADER_STRUCT.unpack(
            header_bytes[:HEADER_BYTES])
        if magic != MAGIC_ZTCP or version != CODEC_VERSION:
            raise ValueError(f"Invalid cold-page header magic/version: {hex(magic)} v{version}")
        return cls(tenant, model, layer, tok, seq, QuantPreset(flags & 0x0F), RoPEMode((flags >> 4) & 0x0F),
                   head_group)


@dataclass(frozen=True)
class ColdPageGeometry:
    """Shape and byte footprint of one KV page (cold_page_spec.py:164-253)."""

    num_tokens: int = 64
    num_kv_heads: int = 8
    head_dim: int = 128
    rope_dim: int = 64
    group_size: int = GROUP_SIZE
    hot_element_bytes: int = 2
    is_mla_single_buffer: bool = False

    def __post_init__(self) -> None:
        if self.head_dim % self.group_size != 0:
            raise ValueError("head_dim must be divisible by group_size")
        if self.rope_dim < 0 or self.rope_dim > self.head_dim:
            raise ValueError("Invalid rope_dim")
        if self.rope_dim % self.group_size != 0:
            raise ValueError("rope_dim must be divisible by group_size")

    @property
    def nope_dim(self) -> int:
        return self.head_dim - self.rope_dim

    @property
    def vectors_per_buffer(self) -> int:
        return self.num_tokens * self.num_kv_heads

    @property
    def hot_page_bytes(self) -> int:
        return (1 if self.is_mla_single_buffer else 2) * self.vectors_per_buffer * self.head_dim * self.hot_element_bytes

    def sections(self, preset: QuantPreset, rope_mode: RoPEMode) -> list[tuple[str, int, int]]:
        """(kind, q_bytes_per_vec, scale_bytes_per_vec) per payload section, in wire order."""
        out = []
        g = self.group_size
        if rope_mode == RoPEMode.PRESERVE_RAW and self.rope_dim > 0:
            out.append(("raw", self.rope_dim * 2, 0))
        elif rope_mode == RoPEMode.PRESERVE_FP8 and self.rope_dim > 0:
            out.append(("int8", self.rope_dim, self.rope_dim // g * 2))
        kq = self.head_dim if rope_mode == RoPEMode.QUANTIZE_ALL else self.nope_dim
        if preset not in (QuantPreset.INT4_SYM, QuantPreset.K8V4_ASYM, QuantPreset.FP8_ONLY):
            raise ValueError(f"Unsupported preset: {preset}")
        if kq > 0:
            out.append(("int4", kq // 2, kq // g * 2) if preset == QuantPreset.INT4_SYM else ("int8", kq, kq // g * 2))
        if not self.is_mla_single_buffer:
            d = self.head_dim
            out.append(("int8", d, d // g * 2) if preset == QuantPreset.FP8_ONLY else ("int4", d // 2, d // g * 2))
        return out

    def min_payload_bytes(self, preset: QuantPreset, rope_mode: RoPEMode) -> int:
        return sum(self.vectors_per_buffer * (q + s) for _, q, s in self.sections(preset, rope_mode))

    def payload_bytes(self, preset: QuantPreset, rope_mode: RoPEMode) -> int:
        """Payload bytes excluding header and tag, padded to a 4-byte multiple."""
        return (self.min_payload_bytes(preset, rope_mode) + 3) // 4 * 4

    def cold_blob_bytes(self, preset: QuantPreset, rope_mode: RoPEMode) -> int:
        return HEADER_BYTES + self.payload_bytes(preset, rope_mode) + TAG_BYTES

    def compression_ratio(self, preset: QuantPreset, rope_mode: RoPEMode) -> float:
        return self.hot_page_bytes / self.cold_blob_bytes(preset, rope_mode)
