"""Builds libtessattn.so in-tree with nvcc for sm_100a.

Usage: python -m tessery_b200.build [--verbose]
The library lands next to this file (tessery_b200/libtessattn.so), where the ctypes
loader looks for it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libtessattn.so"
SOURCES = ["runtime.cu", "simt_kernels.cu", "attn_d32.cu", "attn_d32_tc.cu", "attn_f32_tc.cu", "attn_tc.cu", "attn_short.cu", "noalloc.cu",
           "pool.cu", "linear.cu", "qwen_ops.cu", "qwen3_model.cu",
           "bert_ops.cu", "bert_model.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found; set CUDA_HOME")


def stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    inputs.append(PACKAGE.parent / "include" / "tessattn.h")
    return any(p.stat().st_mtime > built for p in inputs if p.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every CUDA source into one shared library; returns its path."""
    if not force and not stale():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [
        nvcc(),
        *ARCH,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-O3",
        "-shared",
        "-cudart",
        "static",
        "-o",
        str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + result.stdout + result.stderr)
    if verbose:
        sys.stderr.write(result.stdout + result.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(verbose=args.verbose, force=args.force))


if __name__ == "__main__":
    main()
