"""Build recipe for the in-tree C-ABI library ``gdnx_b200/libgdnx.so``.

``python -m gdnx_b200.build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` for sm_100a with nvcc and links one shared library.  Objects go
to ``gdnx_b200/_build/``; the library is written next to this file so it
travels with the source tree.  Rebuilds only what changed (mtime based).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libgdnx.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed ({r.returncode}) on {cmd[-1]}")
    return r.stdout + r.stderr


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header) and not ptxas_info:
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        out = _run(cmd + [str(src)])
        if verbose or ptxas_info:
            sys.stdout.write(out)
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)])
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
    print(LIB)
