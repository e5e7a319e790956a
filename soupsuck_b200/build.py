"""Build libsoupsuck_b200.so in-tree with nvcc for sm_100a (no JIT, no torch extension).

``python -m soupsuck_b200.build`` (or ``__graft_entry__.build()``) compiles the
unity translation unit ``csrc/soupsuck_b200.cu`` into ``_lib/libsoupsuck_b200.so``.
The CUDA runtime is linked statically so the library does not depend on the
runtime version torch ships; streams from torch are passed in as raw handles.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc" / "soupsuck_b200.cu"
OUT = HERE / "_lib" / "libsoupsuck_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the soupsuck_b200 CUDA library cannot be built")


def sources():
    return sorted((HERE / "csrc").glob("*.cu*")) + [HERE.parent / "include" / "soupsuck_b200.h"]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    built = OUT.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-shared", "-cudart", "static", "-o", str(tmp), str(SRC)]
    if verbose:
        cmd.append("-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libsoupsuck_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
