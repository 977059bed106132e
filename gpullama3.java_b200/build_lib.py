"""Builds libgpullama_attn.so for sm_100a with nvcc (in-tree, no JIT cache).

Usage: python gpullama3.java_b200/build_lib.py [--force] [--jobs N]
The shared library lands in gpullama3.java_b200/gpullama_attn/ next to the
ctypes binding that loads it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "gpullama_attn", "libgpullama_attn.so")
INCLUDE = os.path.normpath(os.path.join(HERE, "..", "include"))

SOURCES = ["api.cu", "decode.cu", "combine.cu", "rope.cu", "prefill.cu", "comm.cpp", "peer.cpp",
           "noalloc.cu", "ingest.cu", "wo.cu", "q8.cu", "debug.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(src_paths, target) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(p) > t for p in src_paths)


def _deps() -> list[str]:
    out = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    out.append(os.path.join(INCLUDE, "gpullama_attn.h"))
    return out


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    if not force and not _newer(deps, OUT):
        return OUT
    cc = nvcc()

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD, src + ".o")
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if src.endswith(".cu"):
            cmd.insert(1, "-Xptxas=-v") if verbose else None
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = OUT + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))
