"""Builds libhelix.so (the C-ABI library) in-tree for sm_100a.

Every CUDA source is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -lineinfo``; host sources go through
nvcc's host compiler.  Objects land in helix_b200/_build/, the library in
helix_b200/libhelix.so.  No JIT cache is involved, so the built library
travels with the source tree.

Usage: python -m helix_b200.build [-v] [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libhelix.so"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
          f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("runtime/*.cpp")) + sorted(CSRC.glob("kernels/*.cu"))


def headers() -> list[Path]:
    return (sorted(CSRC.rglob("*.h")) + sorted(CSRC.rglob("*.cuh"))
            + [ROOT / "include" / "helix" / "helix.h"])


def _obj(src: Path) -> Path:
    return BUILD / (src.parent.name + "_" + src.name + ".o")


def _compile(src: Path, verbose: bool) -> Path:
    obj = _obj(src)
    cmd = [NVCC, *COMMON, *ARCH, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"] if verbose else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    newest_hdr = max(p.stat().st_mtime for p in headers())
    todo = [s for s in srcs if force or not _obj(s).exists()
            or _obj(s).stat().st_mtime < max(s.stat().st_mtime, newest_hdr)]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda s: _compile(s, verbose), todo))
    objs = [_obj(s) for s in srcs]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
               "-Xlinker", f"--version-script={CSRC / 'exports.map'}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    out = build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(out)
