"""Build libkdb200.so (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python kernel-development_b200/build.py [--force] [--verbose]

The library is one translation unit (csrc/libkdb200.cu includes every kernel source) compiled by
nvcc for `sm_100a` only, with the CUDA runtime linked statically, into
kernel-development_b200/lib/libkdb200.so.  It is rebuilt when any source under csrc/ or include/ is
newer than the library.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_DIR = PKG_ROOT / "lib"
LIB_PATH = LIB_DIR / "libkdb200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA 12.9 toolkit on PATH)")


def _sources() -> list[Path]:
    srcs = [p for p in CSRC.iterdir() if p.suffix in (".cu", ".cuh", ".h")]
    srcs += [p for p in INCLUDE.iterdir() if p.suffix == ".h"]
    return srcs


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if needed; returns its path.  Raises RuntimeError on a compile error."""
    if not force and not needs_build():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), str(CSRC / "libkdb200.cu")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    (LIB_DIR / "ptxas.log").write_text(log)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{log[-6000:]}")
    if verbose:
        print(log)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    path = build(force=a.force, verbose=a.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
