"""Builds the native library ``lema_b200/liblema_b200.so`` in-tree with nvcc.

Every CUDA source is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); the C++ memory manager is
compiled by nvcc's host compiler into the same shared object. Objects go to
``lema_b200/_build/``; a rebuild happens when any source or header is newer
than the library.

Usage: ``python -m lema_b200.build [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "liblema_b200.so"
INCLUDE_DIR = REPO_DIR / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    f"-I{INCLUDE_DIR}",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build lema_b200")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE_DIR.glob("*.h")))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in sources() + _headers() + [Path(__file__)])


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.name + ".o")
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(f"--- {src.name}\n{r.stdout}{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles and links the library if needed; returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs),
           "-Xlinker", "--no-undefined", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
