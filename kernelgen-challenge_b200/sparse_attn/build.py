"""Build ``libsparse_attn.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m sparse_attn.build`` (from ``kernelgen-challenge_b200/``) or
``sparse_attn.build.build()``.  Sources are ``../csrc/*.cu``; the public
header is ``<repo>/include/sparse_attn.h``.  The library is rebuilt only when a
source or header is newer than it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG_DIR = pathlib.Path(__file__).resolve().parent
SRC_DIR = PKG_DIR.parent / "csrc"
INC_DIR = PKG_DIR.parent.parent / "include"
LIB_PATH = PKG_DIR / "libsparse_attn.so"
OBJ_DIR = PKG_DIR.parent / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
              "-Xptxas", "-v", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: cannot build libsparse_attn.so")
    return cand


def _sources():
    return sorted(SRC_DIR.glob("*.cu"))


def _deps():
    return _sources() + sorted(SRC_DIR.glob("*.cuh")) + sorted(INC_DIR.glob("*.h"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def _compile(src: pathlib.Path) -> tuple[pathlib.Path, str]:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INC_DIR), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and not needs_build():
        return LIB_PATH
    OBJ_DIR.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(_compile, _sources()))
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(o) for o, _ in results]]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
