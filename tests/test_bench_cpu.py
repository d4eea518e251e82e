"""bench.py on CPU: the reference arm prints one JSON line with the contract's keys, from the reference
codec built here (oracle/_ref) or, where that build is absent, the oracle's restatement."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "4",
                          "--warmup", "3", "--cpu-seconds", "0.5"], capture_output=True, text=True, env=env,
                         timeout=300, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run()
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    import bench

    assert d["metric"] == bench.METRIC and d["config"]["workload"] == bench.WORKLOAD


def test_reference_arm_falls_back_to_the_oracle(tmp_path):
    d = _run({"ZTCP_REF_BUILD_DIR": str(tmp_path)})  # an empty build directory: no reference module
    assert d["cpu_baseline"]["kind"] == "port" and d["value"] > 0


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the driver's multi-GPU runs (torchrun, two ranks): rank 0 alone runs the reference codec
    and prints its line; the other rank exits 0 without work."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(port),
                          os.path.join(REPO, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "3",
                          "--warmup", "3", "--cpu-seconds", "0.5"], capture_output=True, text=True, timeout=300,
                         cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
