"""Builds the CUDA library of this package in-tree: csrc/*.cu -> libnemiqmv.so (sm_100a only).

    python -m nemicli_terminal_b200.build        (or __graft_entry__.build())

nvcc cross-compiles without a GPU.  The library links the CUDA runtime statically, so it loads
beside torch without depending on where torch keeps its own runtime.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libnemiqmv.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def sources() -> list:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers() -> list:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.inc"))
                  + glob.glob(os.path.join(HERE, "..", "include", "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in sources() + headers())


def build(force: bool = False, verbose: bool = False, extra: tuple = ()) -> str:
    if not force and up_to_date():
        return LIB_PATH
    cmd = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-cudart", "static", "-o", LIB_PATH + ".tmp", *extra, *sources()]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-4000:]}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra=("-Xptxas", "-v") if "--ptxas" in sys.argv else ()))
