"""Build libhayate_b200.so in-tree with nvcc (sm_100a only).

``python -m hayate_b200.build [--force] [--verbose]`` compiles every
``csrc/*.cu`` to an object under ``_build/`` (in parallel) and links the shared
library next to this file.  Objects are rebuilt when their source or any header
is newer.  ``-Xptxas -v`` output (registers, spills, shared memory) of each
source's latest compile is kept in ``_build/<source>.ptxas.log``, and
``_build/ptxas.log`` is rewritten on every build as their concatenation, so it
always describes the objects the library was linked from.  ``HY_NVCC_DEFINES`` (e.g. ``-DHY_EXP2_POLY_EVERY=2``)
adds preprocessor definitions to every compile, for building a tuning variant
of a kernel constant; rebuild with ``--force`` after changing it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(REPO, "_build")
LIB = os.path.join(PKG, "libhayate_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin directory on PATH")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    defines = os.environ.get("HY_NVCC_DEFINES", "").split()
    cmd = [nvcc(), *ARCH, *FLAGS, *defines, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    todo = [s for s in srcs
            if force or _stale(os.path.join(BUILD, os.path.basename(s)[:-3] + ".o"), [s, *hdrs])]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
                with open(obj[:-2] + ".ptxas.log", "w") as f:
                    f.write(log)
    logs = []
    for src in srcs:
        per = os.path.join(BUILD, os.path.basename(src)[:-3] + ".ptxas.log")
        if os.path.exists(per):
            with open(per) as f:
                logs.append(f"== {os.path.basename(src)[:-3]}.o\n{f.read()}")
    with open(os.path.join(BUILD, "ptxas.log"), "w") as f:
        f.write("\n".join(logs))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    sys.exit(main())
