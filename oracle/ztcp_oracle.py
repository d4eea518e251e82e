"""ctypes binding of the C oracle in ``ztcp_oracle.c`` (test infrastructure only).

The oracle is the parity checker for the CUDA codec.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg may use it; the
product path never imports this module.

Arrays are numpy: fp16 pages as ``uint16`` bit patterns (``[batch, vecs,
head_dim]`` or ``[vecs, head_dim]``), blobs as ``uint8``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ztcp_oracle.c")
LIB_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(LIB_DIR, "libztcp_oracle.so")

HEADER_BYTES = 32
TAG_BYTES = 16


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (IEEE float semantics: no -ffast-math)."""
    if force or not os.path.isfile(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        os.makedirs(LIB_DIR, exist_ok=True)
        subprocess.check_call(
            ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-Wall", "-Wextra", "-o", LIB, SRC, "-lm"]
        )
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.isfile(LIB):
            build()
        L = C.CDLL(LIB)
        u8p, u16p, u32p, u64p, i32p = (C.POINTER(t) for t in (C.c_uint8, C.c_uint16, C.c_uint32, C.c_uint64, C.c_int32))
        L.zo_f32_to_f16.restype = C.c_uint16
        L.zo_f32_to_f16.argtypes = [C.c_float]
        L.zo_f16_to_f32.restype = C.c_float
        L.zo_f16_to_f32.argtypes = [C.c_uint16]
        L.zo_bf16_to_f16.restype = C.c_uint16
        L.zo_bf16_to_f16.argtypes = [C.c_uint16]
        L.zo_chacha20_block.argtypes = [u32p, C.c_uint32, u32p, u8p]
        L.zo_chacha20_xor.argtypes = [u8p, u8p, C.c_size_t, u32p, C.c_uint32, u32p]
        L.zo_siphash128.argtypes = [C.c_uint64, C.c_uint64, u8p, C.c_size_t, u8p]
        L.zo_min_payload_bytes.restype = C.c_int64
        L.zo_min_payload_bytes.argtypes = [C.c_int, C.c_int, C.c_int64, C.c_int64, C.c_int64, C.c_int]
        L.zo_spec_payload_bytes.restype = C.c_int64
        L.zo_spec_payload_bytes.argtypes = L.zo_min_payload_bytes.argtypes
        L.zo_encode_batch.restype = C.c_int
        L.zo_encode_batch.argtypes = [u16p, u16p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int,
                                      C.c_int64, C.c_uint32, C.c_uint32, C.c_uint16, C.c_uint16, u64p, C.c_uint64,
                                      u64p, C.c_uint64, C.c_uint64, u8p]
        L.zo_encode_batch_arith.restype = C.c_int
        L.zo_encode_batch_arith.argtypes = L.zo_encode_batch.argtypes + [C.c_int]
        L.zo_decode_batch.restype = C.c_int64
        L.zo_decode_batch.argtypes = [u8p, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int,
                                      C.c_uint32, C.c_uint32, C.c_uint16, u64p, u64p, C.c_uint64, C.c_uint64,
                                      u16p, u16p, i32p]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def f32_to_f16_bits(x: float) -> int:
    return lib().zo_f32_to_f16(float(x))


def bf16_to_f16_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> fp16 bit patterns, round-to-nearest-even (the reference is fed bf16.half())."""
    f = lib().zo_bf16_to_f16
    flat = np.ascontiguousarray(b, dtype=np.uint16).reshape(-1)
    return np.fromiter((f(int(v)) for v in flat), dtype=np.uint16, count=flat.size).reshape(b.shape)


def chacha20_block(key_words: np.ndarray, counter: int, nonce_words: np.ndarray) -> bytes:
    out = np.zeros(64, np.uint8)
    kw = np.ascontiguousarray(key_words, np.uint32)
    nw = np.ascontiguousarray(nonce_words, np.uint32)
    lib().zo_chacha20_block(_p(kw, C.c_uint32), counter & 0xFFFFFFFF, _p(nw, C.c_uint32), _p(out, C.c_uint8))
    return out.tobytes()


def chacha20_xor(data: bytes, key32: bytes, counter: int, nonce12: bytes) -> bytes:
    src = np.frombuffer(bytes(data), np.uint8).copy()
    dst = np.zeros_like(src)
    kw = np.frombuffer(key32, np.uint32).copy()
    nw = np.frombuffer(nonce12, np.uint32).copy()
    lib().zo_chacha20_xor(_p(src, C.c_uint8), _p(dst, C.c_uint8), src.size, _p(kw, C.c_uint32),
                          counter & 0xFFFFFFFF, _p(nw, C.c_uint32))
    return dst.tobytes()


def siphash24_128(data: bytes, mk0: int, mk1: int) -> bytes:
    src = np.frombuffer(bytes(data), np.uint8).copy()
    out = np.zeros(16, np.uint8)
    lib().zo_siphash128(mk0 & (2**64 - 1), mk1 & (2**64 - 1), _p(src, C.c_uint8), src.size, _p(out, C.c_uint8))
    return out.tobytes()


def min_payload_bytes(preset, rope_mode, vecs, head_dim, rope_dim, has_v) -> int:
    return lib().zo_min_payload_bytes(int(preset), int(rope_mode), vecs, head_dim, rope_dim, int(bool(has_v)))


def spec_payload_bytes(preset, rope_mode, vecs, head_dim, rope_dim, has_v) -> int:
    return lib().zo_spec_payload_bytes(int(preset), int(rope_mode), vecs, head_dim, rope_dim, int(bool(has_v)))


def encode_batch(k_f16: np.ndarray, v_f16: np.ndarray | None, token_hashes, *, rope_dim, preset, rope_mode,
                 expected_payload, tenant, model, layer, head_group, base_seq, key, mac_key,
                 neon: bool = False) -> np.ndarray:
    """Reference batch-egress semantics (page b gets sequence_nonce = base_seq + b).

    k_f16/v_f16: uint16 [batch, tokens, heads, head_dim] (fp16 bits).  Returns uint8 [batch, blob_bytes].
    neon: quantize with the reference's ARM NEON fp16 arithmetic instead of its scalar x86 path.
    """
    k = np.ascontiguousarray(k_f16, np.uint16)
    v = None if v_f16 is None else np.ascontiguousarray(v_f16, np.uint16)
    b, t, h, d = k.shape
    vecs = t * h
    tok = np.ascontiguousarray(np.asarray(token_hashes, dtype=np.uint64))
    keyarr = np.asarray([int(x) & (2**64 - 1) for x in key], np.uint64)
    out = np.zeros((b, HEADER_BYTES + expected_payload + TAG_BYTES), np.uint8)
    rc = lib().zo_encode_batch_arith(_p(k, C.c_uint16), None if v is None else _p(v, C.c_uint16), b, vecs, d,
                                     rope_dim, int(preset), int(rope_mode), expected_payload, tenant & 0xFFFFFFFF,
                                     model & 0xFFFFFFFF, layer & 0xFFFF, head_group & 0xFFFF, _p(tok, C.c_uint64),
                                     base_seq & (2**64 - 1), _p(keyarr, C.c_uint64), int(mac_key[0]) & (2**64 - 1),
                                     int(mac_key[1]) & (2**64 - 1), _p(out, C.c_uint8), int(bool(neon)))
    if rc != 0:
        raise ValueError("oracle encode rejected its arguments")
    return out


def decode_batch(blobs: np.ndarray, token_hashes, *, num_tokens, num_heads, head_dim, rope_dim, is_mla, tenant,
                 model, layer, key, mac_key):
    """Reference batch-ingress semantics.  Returns (k, v|None, status[int32], first_bad_index)."""
    bl = np.ascontiguousarray(blobs, np.uint8)
    b, blob_len = bl.shape
    vecs = num_tokens * num_heads
    tok = np.ascontiguousarray(np.asarray(token_hashes, dtype=np.uint64))
    keyarr = np.asarray([int(x) & (2**64 - 1) for x in key], np.uint64)
    k = np.zeros((b, num_tokens, num_heads, head_dim), np.uint16)
    v = None if is_mla else np.zeros_like(k)
    st = np.zeros(b, np.int32)
    first = lib().zo_decode_batch(_p(bl, C.c_uint8), b, blob_len, vecs, head_dim, rope_dim, int(bool(is_mla)),
                                  tenant & 0xFFFFFFFF, model & 0xFFFFFFFF, layer & 0xFFFF, _p(tok, C.c_uint64),
                                  _p(keyarr, C.c_uint64), int(mac_key[0]) & (2**64 - 1),
                                  int(mac_key[1]) & (2**64 - 1), _p(k, C.c_uint16),
                                  None if v is None else _p(v, C.c_uint16), _p(st, C.c_int32))
    return k, v, st, int(first)
