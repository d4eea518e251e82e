"""Build recipe for the reference codec (test infrastructure only).

Compiles the reference's own C++ codec source, unchanged, from where it lies
in the reference checkout into ``oracle/_ref/`` (git-ignored; the built module
travels with the repository snapshot to GPU boxes, the source does not).  The
result is used in two places only: as a parity checker for the CUDA codec and
the C restatement in ``oracle/ztcp_oracle.c``, and as the timed CPU baseline
(``bench.py --impl reference`` / ``cpu_baseline``).

Flags follow the reference's own JIT build (``native_fused_codec.py:58-64``:
``-O3 -std=c++17 -ffast-math``) with its ARM-only ``-march=armv8.5-a+fp16``
replaced by ``-march=x86-64-v3`` so the module runs on any AVX2 host.  On
x86-64 the reference compiles its scalar (non-NEON) code paths; those are the
paths whose bytes this repository reproduces.

Usage:  python oracle/build_ref.py [--reference-root PATH]
"""
from __future__ import annotations

import argparse
import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.environ.get("ZTCP_REF_BUILD_DIR", os.path.join(HERE, "_ref"))
MODULE_NAME = "ztcp_ref_codec"
REL_SOURCE = os.path.join("research", "baseline_codec", "csrc", "fused_cold_page_cpu.cpp")
DEFAULT_ROOT = os.environ.get("ZTCP_REFERENCE_ROOT",
                              os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))


def built_module_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT_DIR, MODULE_NAME + "*.so")))
    return hits[0] if hits else None


def build(reference_root: str = DEFAULT_ROOT, verbose: bool = False) -> str | None:
    """Compile the reference module if its source is present; return the .so path.

    Returns the already-built module when the source tree is absent (as on a
    GPU box, which only receives the prebuilt file), or None when neither
    exists.
    """
    src = os.path.join(reference_root, REL_SOURCE)
    if not os.path.isfile(src):
        return built_module_path()
    os.makedirs(OUT_DIR, exist_ok=True)
    venv_bin = os.path.dirname(sys.executable)
    if venv_bin not in os.environ.get("PATH", "").split(os.pathsep):
        os.environ["PATH"] = venv_bin + os.pathsep + os.environ.get("PATH", "")
    from torch.utils.cpp_extension import load

    load(
        name=MODULE_NAME,
        sources=[src],
        build_directory=OUT_DIR,
        extra_cflags=["-O3", "-std=c++17", "-ffast-math", "-march=x86-64-v3"],
        verbose=verbose,
    )
    return built_module_path()


def load_module():
    """Import the prebuilt reference module (requires torch in the process)."""
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    path = built_module_path()
    if path is None:
        raise FileNotFoundError(
            "reference codec not built: run `python oracle/build_ref.py` where the reference source is present"
        )
    spec = importlib.util.spec_from_file_location(MODULE_NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=DEFAULT_ROOT)
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.reference_root, verbose=args.verbose))
