"""Build ``libkda_b200.so`` in-tree with nvcc for sm_100a.

``python -m axiom_b200.build`` (or ``build()``) compiles every ``csrc/*.cu``
into ``axiom_b200/libkda_b200.so``.  Objects are cached under ``_build/`` by
source hash, so an unchanged source is not recompiled.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libkda_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--use_fast_math", "-Xcompiler", "-fPIC",
         "-Xptxas", "-O3", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the KDA library needs the CUDA toolkit to build")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    """Every header a source can include: csrc/*.cuh|*.h and include/*.h."""
    out = []
    for d in (CSRC, INCLUDE):
        out += sorted(os.path.join(d, f) for f in os.listdir(d) if f.endswith((".cuh", ".h")))
    return out


def _digest(path: str, extra: str) -> str:
    """Object key: the source, every header (an edit to any of them rebuilds) and the flags."""
    h = hashlib.sha256(extra.encode())
    with open(path, "rb") as f:
        h.update(f.read())
    for p in _headers():
        h.update(os.path.basename(p).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile all CUDA sources and link ``libkda_b200.so``; returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    flags = FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else [])
    key = " ".join(ARCH + flags)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + "." + _digest(src, key) + ".o")
        if os.path.exists(obj) and not ptxas_verbose:
            return obj, ""
        cmd = [nvcc, *ARCH, *flags, "-c", src, "-o", obj]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        return obj, res.stdout + res.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, _sources()))
    objs = [o for o, _ in results]
    if verbose or ptxas_verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    # objects of earlier source versions are never reused once a source changes
    keep = {os.path.basename(o) for o in objs}
    for name in os.listdir(BUILD):
        if name.endswith(".o") and name not in keep:
            os.remove(os.path.join(BUILD, name))
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv))
