"""Compile the oracle's C restatement (routing.c) into oracle/_build/liboracle_routing.so.

TEST INFRASTRUCTURE: the library verifies the GPU routing kernels and is loaded only by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg.

    python oracle/build.py [--force]

No reference sources are compiled here: the reference's code for these paths is either absent
(the OKC problems' reference.py/checks.py) or GPU-only with different math (okc-challenge/engines/*.cu),
so there is no oracle/_ref build.
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "routing.c"
OUT_DIR = HERE / "_build"
LIB = OUT_DIR / "liboracle_routing.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("gcc not found: cannot build the oracle")
    OUT_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-o", str(tmp), str(SRC), "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stdout}{proc.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
