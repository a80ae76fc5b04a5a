"""Build libg4b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python gemma4.c_b200/build.py [--force] [--verbose]

Objects go to gemma4.c_b200/_build/, the library to gemma4.c_b200/libg4b200.so.
No --use_fast_math: the kernels rely on IEEE division/sqrt and on accurate
expf/tanhf/cosf for parity with the reference C path.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libg4b200.so")


def nvcc_path() -> str:
    for p in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if p and os.path.exists(p):
            return p
    raise RuntimeError("nvcc not found")


ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _compile(nvcc: str, src: str, obj: str, verbose: bool) -> str:
    cmd = [nvcc, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, r.stdout, r.stderr))
    return r.stderr


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(HERE, "..", "include", "g4b200.h")]
    objs = []
    jobs = {}
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for s in srcs:
            o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
            objs.append(o)
            if force or verbose or _stale(o, [s, *hdrs]):
                jobs[s] = ex.submit(_compile, nvcc, s, o, verbose)
        for s, f in jobs.items():
            log = f.result()
            if verbose and log:
                sys.stderr.write("== %s\n%s" % (os.path.basename(s), log))
    if force or jobs or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
