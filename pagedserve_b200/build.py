"""Build libpagedserve_b200.so in-tree with nvcc for sm_100a.

    python -m pagedserve_b200.build            # incremental
    python -m pagedserve_b200.build --force    # rebuild everything

Objects go to ``pagedserve_b200/_build/``; the shared library lands next to
this file so it travels with the source tree.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libpagedserve_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps() -> list[str]:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hdrs + [os.path.join(ROOT, "include", "pagedserve_b200.h")]


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(d) for d in _deps()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    extra = list(extra or [])
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(force=a.force, verbose=True)
    sys.exit(0)
