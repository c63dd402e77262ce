"""Compiles the ggml-cuda bridge (ggml-helix-cuda.cpp) against the compile
stand-in in compat/ (not ggml: only the fields the bridge reads), linked to
helix_b200/libhelix.so, into integration/ggml/_build/libggml_helix_cuda.so.

This is how the bridge is compile-checked and exercised in this repository;
a llama.cpp build compiles ggml-helix-cuda.cpp inside ggml-cuda with ggml's
own headers instead.

Usage: python -m integration.ggml.build
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build" / "libggml_helix_cuda.so"


def build() -> Path:
    from helix_b200 import build as hb
    lib = hb.build()
    OUT.parent.mkdir(exist_ok=True)
    cuda = Path(shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc").resolve().parents[1]
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-shared",
           f"-I{HERE / 'compat'}", f"-I{HERE}", f"-I{ROOT / 'include'}", f"-I{cuda / 'include'}",
           str(HERE / "ggml-helix-cuda.cpp"), "-o", str(OUT),
           f"-L{lib.parent}", "-lhelix", f"-Wl,-rpath,{lib.parent}",
           f"-L{cuda / 'lib64'}", "-lcudart", f"-Wl,-rpath,{cuda / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"bridge compile failed\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return OUT


if __name__ == "__main__":
    print(build())
