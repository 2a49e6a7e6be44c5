"""Build the sm_100a shared library ``futudiffu_b200/libfd_b200.so``.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` (relocatable
device code, so the files share the device status word), then device-linked
into one shared object with the CUDA runtime linked statically.  The library
is built in-tree so it travels with the source tree; nothing is installed.

Usage: ``python -m futudiffu_b200.build [--force] [-j N] [--verbose]``
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libfd_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build futudiffu_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


# Files compiled as a whole program (no relocatable device code): ptxas applies
# the per-warp register limits of setmaxnreg only there (the deferred-GELU FP8
# GEMM gives its promotion warps 168 registers out of a 128-per-thread launch).
# Such a file references no other file's device variables (FD_WHOLE_PROGRAM).
WHOLE_PROGRAM = {"gemm_fp8.cu"}


def _flags(src: Path) -> list[str]:
    if src.name in WHOLE_PROGRAM:
        return [f for f in NVCC_FLAGS if f != "-rdc=true"] + ["-DFD_WHOLE_PROGRAM"]
    return NVCC_FLAGS


def _compile(src: Path, verbose: bool, force: bool, hmtime: float) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hmtime):
        return obj
    cmd = [nvcc(), *ARCH, *_flags(src), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile all kernels and link ``libfd_b200.so``; returns its path."""
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    hmtime = _headers_mtime()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, force, hmtime), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not force and LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-rdc=true", "-cudart", "static", *map(str, objs), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, jobs=a.jobs, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
