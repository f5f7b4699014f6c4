"""Build libs4mm.so (all CUDA sources, sm_100a) in-tree with nvcc.

Called by ``__graft_entry__.build()`` and by the package-level ``build()``. Objects go to
``_build/`` beside this file; the shared library is
written next to this file so that it travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libs4mm.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the s4mm CUDA library cannot be built")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h", ".inc"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, extra) -> str:
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False, extra=()) -> str:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libs4mm.so``. Returns the library path."""
    os.makedirs(OBJ, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, list(extra)), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print("built", LIB)
    return LIB


def ptxas_report(src_name: str) -> str:
    """``-Xptxas -v`` register/shared-memory report of one source (for tuning notes)."""
    src = os.path.join(CSRC, src_name)
    cmd = [nvcc(), *ARCH, *FLAGS, "-Xptxas", "-v", "-c", src, "-o", os.devnull]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.stdout + r.stderr


if __name__ == "__main__":
    build(verbose=True)
