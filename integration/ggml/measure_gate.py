"""Measures the bridge's length gate on a B200: per call, the time of HELIX's
chunked scan (through helix_scan_encode with the bridge's own descriptor:
F32 tensors, no dt clamp, multipass; the default fp32 kernels and the
GGML_HELIX_BF16 tensor-core path) against a plain per-token scan kernel
(gate/per_token_scan.cu, the kind of kernel a framework runs when HELIX
declines), for growing token counts.  The smallest length from which HELIX
is faster is the crossover; the bridge's default minimum sits at or above it.

The per-token kernel is first checked against the fp64 oracle.  Timing is
GPU time: a long fill is queued first so that the host has issued all 50
calls before the GPU reaches them, and CUDA events around the 50 calls give
the per-call mean of back-to-back execution -- host issue costs are left
out, as a framework's CUDA graph leaves them out.

Usage: python -m integration.ggml.measure_gate [--heads 48] [--json out.json]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

LENGTHS = [1, 4, 8, 16, 24, 32, 48, 64, 96, 128, 256, 512, 1024, 2048]


def build_baseline() -> Path:
    out = HERE / "_build" / "libper_token_scan.so"
    out.parent.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    src = HERE / "gate" / "per_token_scan.cu"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        subprocess.run([nvcc, "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
                        "-shared", str(src), "-o", str(out)], check=True)
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--heads", type=int, default=48)
    ap.add_argument("--json", default="")
    a = ap.parse_args()
    import numpy as np
    import torch

    import helix_b200
    from helix_b200 import abi
    from helix_b200.synth import Shape, make_inputs
    from oracle.oracle import Oracle

    lib = C.CDLL(str(build_baseline()))
    lib.per_token_scan.argtypes = [C.c_int] * 6 + [C.c_void_p] * 8 + [C.c_void_p]
    lib.per_token_scan.restype = C.c_int
    dev = torch.device("cuda:0")
    ctx = helix_b200.Context(0)
    stream = torch.cuda.Stream(dev)
    H, P, N, G = a.heads, 64, 128, 1

    def inputs(L):
        t = make_inputs(Shape(1, L, H, P, N, G, "f32"), seed=7, device=dev, s0_std=0.1)
        t["y"] = torch.empty(t["x"].shape, device=dev)
        t["s1"] = torch.empty_like(t["s0"])
        return t

    def per_token(t, L):
        rc = lib.per_token_scan(1, L, H, P, N, G, *[t[k].data_ptr() for k in ("x", "dt", "A", "B", "C", "s0",
                                                                                   "y", "s1")], stream.cuda_stream)
        assert rc == 0, rc
        return rc

    # the baseline is a correct scan
    L0 = 300
    t = inputs(L0)
    torch.cuda.synchronize()
    assert per_token(t, L0) == 0
    torch.cuda.synchronize()
    o = Oracle()
    d = o.desc_init(L0, 1, H, P, N, G)
    d.dt_max = float("inf")
    ref_y, ref_s = o.scan(d, *[t[k].cpu().numpy() for k in ("s0", "x", "dt", "A", "B", "C")])
    for got, want in ((t["y"], ref_y), (t["s1"], ref_s)):
        g = got.cpu().numpy().astype(np.float64)
        err = float(np.linalg.norm(g - want) / np.linalg.norm(want))
        assert err < 1e-5, err

    hold = torch.empty(1 << 30, dtype=torch.uint8, device=dev)

    def timed(fn, calls=50):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(4):
                hold.fill_(1)  # keeps the GPU busy while the calls are issued
        e0.record(stream)
        for _ in range(calls):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / calls  # us per call

    rows = []
    for L in LENGTHS:
        t = inputs(L)
        res = {"L": L, "per_token_us": timed(lambda: per_token(t, L))}
        for name, compute in (("helix_f32_us", "f32"), ("helix_bf16_us", "bf16")):
            dd = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], t["y"], multipass=True,
                                              compute=compute)
            dd.dt_max = float("inf")
            n = ctx.scratch_size(dd)
            scratch = torch.empty(max(n, 256), dtype=torch.uint8, device=dev)

            def call():
                st = ctx.encode(dd, t["s0"], t["x"], t["dt"], t["A"], t["B"], t["C"], t["y"], t["s1"],
                                scratch=scratch, stream=stream)
                assert st == abi.HELIX_OK, ctx.last_error()
            res[name] = timed(call)
        rows.append(res)
        print(json.dumps(res), flush=True)

    def crossover(key):
        for r in rows:
            if all(q[key] < q["per_token_us"] for q in rows if q["L"] >= r["L"]):
                return r["L"]
        return None
    summary = {"heads": H, "head_dim": P, "d_state": N, "groups": G,
               "crossover_f32": crossover("helix_f32_us"), "crossover_bf16": crossover("helix_bf16_us"),
               "rows": rows}
    print(json.dumps({k: v for k, v in summary.items() if k != "rows"}))
    if a.json:
        Path(a.json).write_text(json.dumps(summary, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
