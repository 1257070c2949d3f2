"""Builds libqb_gdn.so (the C ABI of include/qb_gdn.h) in-tree with nvcc for sm_100a.

    python -m quotebound_b200.build [--force] [--verbose]

Every .cu under csrc/ is compiled to an object in csrc/_build/ (in parallel) and linked into
quotebound_b200/libqb_gdn.so, which carries no torch symbols: any C/C++ host can dlopen it.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(CSRC, "_build")
LIB = os.path.join(HERE, "libqb_gdn.so")
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def _deps(src: str) -> list[str]:
    return [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, extra: list[str]) -> str:
    obj = os.path.join(OBJ, os.path.basename(src).replace(".cu", ".o"))
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile and link libqb_gdn.so if any source changed; returns its path."""
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    todo = [s for s in sources
            if force or _stale(os.path.join(OBJ, os.path.basename(s).replace(".cu", ".o")), _deps(s))]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda s: _compile(s, verbose, extra or []), todo))
    objs = [os.path.join(OBJ, os.path.basename(s).replace(".cu", ".o")) for s in sources]
    if force or todo or _stale(LIB, objs):
        # the CUDA runtime is linked statically (nvcc's default): the library needs only the driver
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


def ensure() -> str:
    """The library, building it only if it is missing (a shipped build is used as is)."""
    return LIB if os.path.exists(LIB) else build()


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
