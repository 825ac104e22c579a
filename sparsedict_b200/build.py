"""Build libsparsedict_b200.so in-tree with nvcc for sm_100a.

    python -m sparsedict_b200.build [--force]

The shared library lands next to this file so that it travels with the
source tree; nothing is installed elsewhere.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libsparsedict_b200.so"
SOURCES = ["capi.cu", "fwd_generic.cu", "fwd_tc.cu", "bwd.cu", "bwd_km.cu", "stages.cu", "select_attn.cu",
           "bwd_noalloc.cu", "affinity_tc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps += list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > built for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", *ARCH, f"-I{ROOT / 'include'}"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmd = [nvcc(), *flags, "-c", str(CSRC / src), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    sys.exit(0)
