"""Build libneedle_b200.so (sm_100a) in-tree.

    python needle-rs_b200/build.py [--force] [--verbose-ptxas]

Every CUDA source compiles for sm_100a only (`-gencode arch=compute_100a,
code=sm_100a`); the library links the CUDA runtime statically so it carries no
dependency beyond the driver. Output: needle-rs_b200/lib/libneedle_b200.so.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libneedle_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".hpp", ".h"))]
    hs.append(os.path.join(os.path.dirname(HERE), "include", "needle.h"))
    return hs


def _compile(src, ptxas_verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, obj, r


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sources()
    hdr_m = max(os.path.getmtime(h) for h in headers())
    todo = []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s) + ".o")
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(s), hdr_m):
            todo.append(s)
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(todo)))) as ex:
        for src, obj, r in ex.map(lambda s: _compile(s, ptxas_verbose), todo):
            logs.append(r.stderr)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed on {os.path.basename(src)}")
            if not quiet and r.stderr:
                sys.stderr.write(r.stderr)
    objs = [os.path.join(BUILD, os.path.basename(s) + ".o") for s in srcs]
    if todo or not os.path.exists(LIB):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libneedle_b200.so failed")
    if ptxas_verbose:
        with open(os.path.join(BUILD, "ptxas.log"), "w") as f:
            f.write("\n".join(logs))
    return LIB


if __name__ == "__main__":
    lib = build(force="--force" in sys.argv, ptxas_verbose="--verbose-ptxas" in sys.argv, quiet=False)
    print(lib)
