"""Shared test helpers: golden-vector loading and input regeneration."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_json(name: str):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def small_cases():
    """(case dict, arrays) for every case of codec_small.npz."""
    cases = load_json("codec_small.json")
    arrays = np.load(os.path.join(GOLDEN, "codec_small.npz"))
    return cases, arrays


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def full_case_inputs(case: dict):
    """Regenerate a codec_digests.json case's inputs: (k_bf16, v_bf16|None, k16, v16|None, material, toks, shape)."""
    import torch

    from ztcp_b200 import workload

    shape = getattr(workload, case["shape"])
    k32, v32 = workload.kv_pages_np(case["pages"], shape, seed=case["seed"])
    kb = torch.from_numpy(k32).to(torch.bfloat16)
    vb = None if v32 is None else torch.from_numpy(v32).to(torch.bfloat16)
    k16 = kb.half()
    v16 = None if vb is None else vb.half()
    m = workload.session_material(seed=case["seed"])
    toks = workload.token_hashes(case["pages"], seed=case["seed"] + 1)
    return kb, vb, k16, v16, m, toks, shape


def oracle_encode(oracle, k16: np.ndarray, v16, toks, rope_dim, preset, rope_mode, exp, m):
    return oracle.encode_batch(k16.view(np.uint16), None if v16 is None else v16.view(np.uint16),
                               np.asarray(toks).view(np.uint64), rope_dim=rope_dim, preset=preset,
                               rope_mode=rope_mode, expected_payload=exp, tenant=m["tenant"], model=m["model"],
                               layer=m["layer"], head_group=m["head_group"], base_seq=m["base_seq"], key=m["key"],
                               mac_key=m["mac_key"])


def oracle_decode(oracle, blobs, toks, shape4, rope_dim, mla, m):
    T, H, D = shape4[1:]
    return oracle.decode_batch(blobs, np.asarray(toks).view(np.uint64), num_tokens=T, num_heads=H, head_dim=D,
                               rope_dim=rope_dim, is_mla=mla, tenant=m["tenant"], model=m["model"],
                               layer=m["layer"], key=m["key"], mac_key=m["mac_key"])


def attention_output_cosine(k_ref, v_ref, k_hat, v_hat, n_queries: int = 32, seed: int = 99) -> float:
    """The reference benchmark's fidelity metric (bench:97-146); see ztcp_b200.workload.attention_cosine."""
    from ztcp_b200 import workload

    return workload.attention_cosine(k_ref, v_ref, k_hat, v_hat, n_queries=n_queries, seed=seed)
