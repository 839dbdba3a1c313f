"""Build liblumina_cuda.so in-tree for sm_100a with nvcc.

    python lumina-studio_b200/build.py [--force] [--verbose]

Objects go to lumina-studio_b200/_build/, the library to
lumina-studio_b200/lumina_b200/liblumina_cuda.so (found there by the ctypes
binding; override with LUMINA_CUDA_LIB). Incremental on source mtimes.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "lumina_b200", "liblumina_cuda.so")
INCLUDE = os.path.join(REPO, "include")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def run(cmd, verbose):
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("command failed: " + " ".join(cmd[:3]) + " ...")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr)
    return r


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = os.environ.get("NVCC", "nvcc")
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    newest_hdr = max(os.path.getmtime(h) for h in hdrs)
    objs = []
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
                    "-I", INCLUDE, "-I", CSRC, "--expt-relaxed-constexpr"]
    if os.environ.get("LUMINA_PTXAS_VERBOSE"):
        flags += ["-Xptxas", "-v"]
    todo = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if (not force and os.path.exists(o) and os.path.getmtime(o) > os.path.getmtime(s)
                and os.path.getmtime(o) > newest_hdr):
            continue
        todo.append((s, o))
    # translation units compile in parallel (the per-bit GEMV units dominate)
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 4))) as ex:
        for r in ex.map(lambda so: run([nvcc, "-c", so[0], "-o", so[1]] + flags, verbose), todo):
            if os.environ.get("LUMINA_PTXAS_VERBOSE"):
                sys.stdout.write(r.stderr)
    if force or not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        run([nvcc, "-shared", "-o", OUT] + objs + ARCH, verbose)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
