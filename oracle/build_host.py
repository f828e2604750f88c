"""Build the C restatement (``sa_host.c``) into ``oracle/_build/libsa_host.so``.

TEST INFRASTRUCTURE ONLY: the library is the second CPU oracle and the timed
CPU baseline; the product library never loads it.  Plain ``gcc`` with OpenMP,
no architecture-specific flags (the library travels to other hosts).
"""
from __future__ import annotations

import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
SRC = HERE / "sa_host.c"
OUT = HERE / "_build" / "libsa_host.so"


def build_host(force: bool = False) -> pathlib.Path:
    if not force and OUT.exists() and OUT.stat().st_mtime >= max(
            SRC.stat().st_mtime, (HERE.parent / "include" / "sparse_attn_host.h").stat().st_mtime):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["gcc", "-O3", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-Wall", "-Werror",
           str(SRC), "-o", str(OUT), "-lm"]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build_host(force=True))
