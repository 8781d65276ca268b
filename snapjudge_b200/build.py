"""Build the B200 extension library in-tree: ``snapjudge_b200/lib/libsnapjudge_b200.so``.

Every ``csrc/*.cu`` is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with line info, then linked into
one shared library with the static CUDA runtime.  Objects are cached by
content hash under ``snapjudge_b200/lib/obj`` so rebuilding after an edit
recompiles only the changed units.  nvcc cross-compiles: no GPU is needed.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libsnapjudge_b200.so")
ROOT = os.path.dirname(HERE)

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _hash(path: str, extra: list[str]) -> str:
    h = hashlib.sha1()
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cuh", ".h")):
            with open(os.path.join(CSRC, f), "rb") as fh:
                h.update(fh.read())
    with open(os.path.join(ROOT, "include", "snapjudge_b200.h"), "rb") as fh:
        h.update(fh.read())
    with open(path, "rb") as fh:
        h.update(fh.read())
    h.update(" ".join(extra).encode())
    return h.hexdigest()[:16]


def _compile(src: str, verbose: bool) -> str:
    path = os.path.join(CSRC, src)
    obj_dir = os.path.join(LIB_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    obj = os.path.join(obj_dir, f"{src[:-3]}.{_hash(path, ARCH + FLAGS)}.o")
    if not os.path.exists(obj):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj + ".tmp"]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, file=sys.stderr)
        os.replace(obj + ".tmp", obj)
    return obj


def build(verbose: bool = False) -> str:
    """Compile and link the library; returns its path."""
    os.makedirs(LIB_DIR, exist_ok=True)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), _sources()))
    # drop cached objects of sources that no longer exist in this form
    keep = {os.path.basename(o) for o in objs}
    obj_dir = os.path.join(LIB_DIR, "obj")
    for f in os.listdir(obj_dir):
        if f.endswith(".o") and f not in keep:
            os.remove(os.path.join(obj_dir, f))
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
