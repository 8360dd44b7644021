"""Build recipe of the product library: libfufft_b200.so for sm_100a.

    python -m fufft_b200.build [-j JOBS] [--verbose]

Every .cu under csrc/ compiles in parallel with nvcc (-gencode
arch=compute_100a,code=sm_100a, -O3 -lineinfo), then the objects link into
one shared library next to this file.  The library has a plain C ABI
(include/fufft_b200.h) and links only the CUDA runtime.  Rebuilds only what
changed (object newer than every source and header).
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
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfufft_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _newest_dep() -> float:
    deps = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max(os.path.getmtime(p) for p in deps)


def _compile(src: str, extra: list[str]) -> tuple[str, str]:
    obj = os.path.join(OBJ, os.path.basename(src).replace(".cu", ".o"))
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + extra + ["-I", INCLUDE, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr[-6000:]}")
    return obj, r.stderr


def build(jobs: int | None = None, verbose: bool = False, extra: list[str] | None = None,
          force: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    extra = extra or []
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    newest = _newest_dep()
    todo = [s for s in srcs if force or not os.path.exists(os.path.join(OBJ, os.path.basename(s)[:-3] + ".o"))
            or os.path.getmtime(os.path.join(OBJ, os.path.basename(s)[:-3] + ".o")) < newest]
    logs = {}
    if todo:
        with cf.ThreadPoolExecutor(jobs or os.cpu_count()) as ex:
            for obj, log in ex.map(lambda s: _compile(s, extra), todo):
                logs[obj] = log
    objs = [os.path.join(OBJ, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        subprocess.run(cmd, check=True)
    if verbose:
        for obj, log in logs.items():
            print(f"== {os.path.basename(obj)}\n{log}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    t = build(a.jobs, a.verbose, force=a.force)
    print(t)
