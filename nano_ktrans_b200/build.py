"""Build ``libmoe_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m nano_ktrans_b200.build [--verbose]``.  Object files go to
``nano_ktrans_b200/_build/``; the shared library lands next to this file so it
travels with the source tree.  The library is rebuilt whenever the SHA-256 of
its sources, headers and compiler flags differs from the digest recorded
beside it when it was built (``libmoe_b200.so.srchash``): a library built from
other sources is never reused, whatever the file times say.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmoe_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmoe_b200.so")
    return path


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


STAMP = LIB + ".srchash"


def source_digest() -> str:
    """SHA-256 over the compiler flags and every source and header, by name and content."""
    h = hashlib.sha256()
    h.update(" ".join(ARCH + FLAGS[:-1]).encode())  # the include path itself is machine-specific
    for p in sorted(_deps()):
        h.update(os.path.relpath(p, os.path.dirname(PKG)).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def up_to_date() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return False
    with open(STAMP) as f:
        return f.read().strip() == source_digest()


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr}")
        if ptxas_info or verbose:
            sys.stderr.write(res.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    with open(STAMP, "w") as f:
        f.write(source_digest() + "\n")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, ptxas_info=a.ptxas_info))
