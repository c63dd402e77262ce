"""Builds the test-only native probes under tests/native (sm_100a)."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def build() -> Path:
    src = HERE / "umma_probe.cu"
    out = HERE / "libumma_probe.so"
    dep = [src, ROOT / "helix_b200/csrc/kernels/umma.cuh"]
    if out.exists() and out.stat().st_mtime >= max(p.stat().st_mtime for p in dep):
        return out
    cmd = [NVCC, "-std=c++17", "-O2", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
           "-Xcompiler", "-fPIC", "-shared", f"-I{ROOT / 'helix_b200/csrc'}", str(src), "-o", str(out)]
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    print(build())
