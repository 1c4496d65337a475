"""Builds the in-tree CUDA library ``littlellm_b200/libkllm_b200.so``.

Every ``csrc/*.cu`` file is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with nvcc and linked into one
shared library exporting the C ABI of ``include/kllm_b200.h``. The CUDA
runtime is linked statically, so the library only needs the driver at run
time. Rebuilds are incremental on source / header modification times.

    python -m littlellm_b200.build [--force] [--verbose]
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
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ_DIR = os.path.join(PKG, "_build")
LIB_PATH = os.path.join(PKG, "libkllm_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-Wall",
    "-I", INCLUDE, "-I", CSRC, "--threads", "2",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libkllm_b200.so")
    return path


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compiles and links the library; returns its path."""
    headers = _headers()
    if not force and not _stale(LIB_PATH, _sources() + headers):
        return LIB_PATH
    os.makedirs(OBJ_DIR, exist_ok=True)
    jobs = []
    for src in _sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        if force or _stale(obj, [src] + headers):
            cmd = [nvcc(), *NVCC_FLAGS, "-c", src, "-o", obj]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            jobs.append((src, cmd))
    objs = [os.path.join(OBJ_DIR, os.path.basename(s)[:-3] + ".o") for s in _sources()]

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        return src, res

    if jobs:
        workers = min(len(jobs), max(1, (os.cpu_count() or 2)))
        with cf.ThreadPoolExecutor(workers) as ex:
            for src, res in ex.map(run, jobs):
                if res.returncode != 0:
                    sys.stderr.write(res.stdout + res.stderr)
                    raise RuntimeError(f"nvcc failed on {os.path.basename(src)}")
                if verbose or ptxas_info:
                    sys.stderr.write(res.stderr)
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("linking libkllm_b200.so failed")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills per kernel")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
