"""Build libunicache_b200.so (the C-ABI library) for sm_100a with nvcc.

Every ``csrc/*.cu`` file is compiled to an object (in parallel) and linked into
``unicache_b200/_lib/libunicache_b200.so`` with the static CUDA runtime, so the
library has no dependency on the CUDA toolkit that PyTorch bundles.  The build
is incremental: an object is rebuilt only when its source or a header changed.

    python -m unicache_b200.build [--force] [--verbose-ptxas]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
BUILD_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libunicache_b200.so")
HEADERS = [os.path.join(ROOT, "include", "unicache_b200.h")] + glob.glob(os.path.join(CSRC, "*.cuh"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    # IEEE division/sqrt and no FMA contraction surprises in the bit-exact
    # quantizer: the kernels use explicit __f*_rn intrinsics where it matters.
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build unicache_b200")
    return path


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *HEADERS])


def _compile(src: str, force: bool, ptxas_verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD_DIR, os.path.basename(src).replace(".cu", ".o"))
    if not force and not _stale(obj, src):
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(BUILD_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        results = list(pool.map(lambda s: _compile(s, force, ptxas_verbose), sources))
    objects = [obj for obj, _ in results]
    if ptxas_verbose and not quiet:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objects):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objects]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    if not quiet:
        print(f"built {LIB}")
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    args = parser.parse_args()
    build(force=args.force, ptxas_verbose=args.verbose_ptxas)


if __name__ == "__main__":
    main()
