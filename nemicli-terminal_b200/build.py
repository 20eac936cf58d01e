"""Builds the CUDA library of this package in-tree: csrc/*.cu -> libnemiqmv.so (sm_100a only).

    python -m nemicli_terminal_b200.build        (or __graft_entry__.build())

nvcc cross-compiles without a GPU.  The sources compile to separate objects in parallel: qmv_fmt.cu once
per block format (-DQMV_FMT_ID=<GGML type id>), every other .cu once; an object is rebuilt only when its
source or a header is newer.  The library links the CUDA runtime statically, so it loads beside torch
without depending on where torch keeps its own runtime.
"""
from __future__ import annotations

import concurrent.futures as cf
import fcntl
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libnemiqmv.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
OBJ_DIR = os.path.join(HERE, "_build")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
PER_FORMAT = "qmv_fmt.cu"


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


def format_ids() -> list:
    """GGML type ids of the formats with kernels (formats.py is the one list)."""
    sys.path.insert(0, HERE)
    try:
        import importlib.util
        spec = importlib.util.spec_from_file_location("_qmv_formats", os.path.join(HERE, "formats.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        sys.path.pop(0)
    return sorted(mod.TYPE_ID.values())


def units(obj_dir: str) -> list:
    """(source, object, extra defines) of every object of the library."""
    out = []
    for src in sources():
        base = os.path.splitext(os.path.basename(src))[0]
        if os.path.basename(src) == PER_FORMAT:
            for fid in format_ids():
                out.append((src, os.path.join(obj_dir, f"{base}_{fid}.o"), [f"-DQMV_FMT_ID={fid}"]))
        else:
            out.append((src, os.path.join(obj_dir, f"{base}.o"), []))
    return out


def _deps(obj: str):
    """Headers the object was compiled from (nvcc -MD writes them next to it), or None if unknown."""
    try:
        text = open(obj + ".d").read().replace("\\\n", " ")
    except OSError:
        return None
    parts = text.split(":", 1)
    return [p for p in parts[1].split()] if len(parts) == 2 else None


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    if os.path.getmtime(src) > t:
        return True
    deps = _deps(obj)
    if deps is None:
        return newest_header > t
    return any(not os.path.exists(d) or os.path.getmtime(d) > t for d in deps)


def up_to_date(out: str = LIB_PATH, obj_dir: str = OBJ_DIR) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(p) <= t for p in sources() + headers())


def build(force: bool = False, verbose: bool = False, extra: tuple = (), out: str = LIB_PATH,
          obj_dir: str = OBJ_DIR, jobs: int = 0) -> str:
    """Compile the stale objects in parallel and link `out`.  extra: more nvcc flags (e.g. -D...).
    Processes that build at the same time (one per rank under torchrun) take turns on a lock file in
    obj_dir; the later ones find the library up to date."""
    if not force and up_to_date(out, obj_dir):
        return out
    os.makedirs(obj_dir, exist_ok=True)
    with open(os.path.join(obj_dir, ".lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and up_to_date(out, obj_dir):
            return out
        return _build_locked(force, verbose, extra, out, obj_dir, jobs)


def _build_locked(force: bool, verbose: bool, extra: tuple, out: str, obj_dir: str, jobs: int) -> str:
    stamp = os.path.join(obj_dir, "flags.txt")
    flags = " ".join(extra)
    if not os.path.exists(stamp) or open(stamp).read() != flags:
        force = True                                   # other flags: every object is stale
    newest = max(os.path.getmtime(p) for p in headers())
    todo = [u for u in units(obj_dir) if force or _stale(u[0], u[1], newest)]
    base = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", *extra]

    def compile_one(u):
        src, obj, defs = u
        cmd = [*base, *defs, "-MD", "-MF", obj + ".d", "-c", "-o", obj + ".tmp", src]
        if verbose:
            print(" ".join(cmd), file=sys.stderr, flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)} {defs} ({res.returncode}):\n"
                               f"{res.stderr[-4000:]}")
        if verbose and res.stderr:
            print(res.stderr, file=sys.stderr, flush=True)
        os.replace(obj + ".tmp", obj)

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        for f in [ex.submit(compile_one, u) for u in todo]:
            f.result()
    with open(stamp, "w") as f:
        f.write(flags)
    objs = [u[1] for u in units(obj_dir)]
    cmd = [nvcc(), *ARCH_FLAGS, "--shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-o", out + ".tmp", *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed ({res.returncode}):\n{res.stderr[-4000:]}")
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra=("-Xptxas", "-v") if "--ptxas" in sys.argv else ()))
