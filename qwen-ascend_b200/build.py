"""Build ``fnx/libfnx_b200.so`` from ``csrc/`` for sm_100a (nvcc cross-compiles; no GPU
needed).  Usage: ``python qwen-ascend_b200/build.py [--force]``."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
OUT = HERE / "fnx" / "libfnx_b200.so"
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static"]


def stale() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SRC.iterdir() if p.suffix in (".cu", ".cuh", ".h"))


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return OUT
    cmd = [NVCC, *FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-I", str(SRC), "-I", str(HERE.parent / "include"),
           "-o", str(OUT) + ".tmp", str(SRC / "fnx_b200.cu")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed ({r.returncode}): {' '.join(cmd)}")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
