"""Build libattn_b200.so in-tree with nvcc for sm_100a.

    python llm-gpu-5_b200/build.py            # incremental
    python llm-gpu-5_b200/build.py --clean    # rebuild everything

Every ``csrc/*.cu`` is compiled separately (objects under ``_build/``, which is not committed)
and linked into ``libattn_b200.so`` beside this file.  The CUDA runtime is linked statically;
the CUDA driver API is reached through ``cudaGetDriverEntryPoint`` at run time, so the library
needs no ``libcuda`` at link time and builds on a machine without a GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(os.path.dirname(PKG), "_build")
LIB = os.path.join(PKG, "libattn_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime(src):
    """Newest mtime of the source and the headers it may include."""
    t = os.path.getmtime(src)
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".cuh", ".h")):
                t = max(t, os.path.getmtime(os.path.join(d, f)))
    return t


def _compile(nvcc, src, obj, verbose):
    cmd = [nvcc, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose else ""


def build(clean=False, verbose=False, jobs=None):
    nvcc = _nvcc()
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    todo = []
    objs = []
    for f in srcs:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f[:-3] + ".o")
        objs.append(obj)
        if clean or not os.path.exists(obj) or os.path.getmtime(obj) < _deps_mtime(src):
            todo.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        for out in ex.map(lambda so: _compile(nvcc, so[0], so[1], verbose), todo):
            if out:
                sys.stderr.write(out)
    newest = max(os.path.getmtime(o) for o in objs)
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill usage")
    a = ap.parse_args()
    print(build(clean=a.clean, verbose=a.verbose))
