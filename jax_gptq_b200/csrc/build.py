"""Build ``jax_gptq_b200/libgq.so`` from the CUDA sources in this directory.

    python -m jax_gptq_b200.csrc.build [--force] [--jobs N]

Every ``*.cu`` file is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) into ``jax_gptq_b200/_build/`` and linked
into one shared library next to the package.  Compilation runs in parallel
and is skipped for objects newer than their sources and headers.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libgq.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", os.path.join(ROOT, "include"), "-I", HERE]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgq")


def _headers() -> list[str]:
    return glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(obj: str, src: str, headers: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *headers])


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    headers = _headers()
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, src, headers):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr}")
        return res.stderr

    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for out in ex.map(compile_one, todo):
            if verbose and out:
                print(out)
    if todo or force or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.force, args.jobs, args.verbose))


if __name__ == "__main__":
    main()
