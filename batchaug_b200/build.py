"""Build libbatchaug_b200.so in-tree for sm_100a.

    python batchaug_b200/build.py [--force] [--jobs N]

Each ``csrc/*.cu`` is compiled separately (in parallel) to an object under
``batchaug_b200/_build/`` and the objects are linked into
``batchaug_b200/libbatchaug_b200.so`` with the CUDA runtime linked statically,
so the library has no dependency on a particular libcudart.  Every file is
compiled with ``-fmad=false``: the kernels reproduce torch's CPU rounding, and
fused multiply-adds appear only where the source asks for them.
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
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbatchaug_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-v",
    "-I" + os.path.join(ROOT, "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the batchaug_b200 CUDA library cannot be built")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [
        os.path.join(ROOT, "include", "batchaug_b200.h")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(nvcc: str, src: str, force: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and not _stale(obj, [src] + _headers() + [__file__]):
        return obj, ""
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{p.stdout}\n{p.stderr}")
    return obj, p.stderr


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    """Compile every kernel for sm_100a and link the shared library."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda s: _compile(nvcc, s, force), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stdout}\n{p.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))
