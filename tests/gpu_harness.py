"""GPU-side helpers for the parity tests: upload numpy problems, run the scan
through the C ABI (helix_scan_encode via ctypes), download results."""
from __future__ import annotations

import json
import os

import numpy as np

import helix_b200
from helix_b200 import abi

# fp32 path: the reference's calibrated per-element bound for its fp32 kernel
# (reference tests/test_metal_parity.mm:35-38) and the north star's 1e-4
# relative L2 for the fp32 path.
F32_REL, F32_ABS, F32_RL2 = 5e-6, 5e-7, 1e-4
# fp32-class tensor-core path (every fp32 operand as a bf16 hi + lo pair,
# three products): the north star's 1e-4 relative L2 for the fp32 path, and
# ten times the reference's fp32 per-element bound (this family measures
# 4-7e-6 relative L2 and up to ~5x that per-element bound on the reference's
# shape matrix).
X3_REL, X3_ABS, X3_RL2 = 5e-5, 5e-6, 1e-4
# bf16-operand path: the reference's calibrated bf16 bound (same file) and the
# north star's 2e-2 relative L2.
BF16_REL, BF16_ABS, BF16_RL2 = 1.5e-2, 3e-3, 2e-2


def record(tag: str, **kv):
    """Appends measured error statistics to $HELIX_TEST_STATS (if set)."""
    path = os.environ.get("HELIX_TEST_STATS")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"tag": tag, **kv}) + "\n")


def run(ctx, prob: dict, *, multipass=True, backend=abi.HELIX_BACKEND_AUTO, compute="auto",
        io="f32", ids=None, desc_hook=None, stream=None, device="cuda:0", y_view=None):
    """prob: numpy float32 arrays s0, x, dt, A, B, C in dense helix.h layouts.
    y_view(shape, device), if given, returns the (possibly strided) y tensor
    the scan writes."""
    import torch
    dev = torch.device(device)
    io_t = torch.bfloat16 if io == "bf16" else torch.float32
    t = {k: torch.from_numpy(np.ascontiguousarray(prob[k])).to(dev) for k in ("s0", "x", "dt", "A", "B", "C")}
    for k in ("x", "B", "C"):
        t[k] = t[k].to(io_t)
    if y_view is None:
        y = torch.full(t["x"].shape, float("nan"), dtype=torch.float32, device=dev)
    else:
        y = y_view(t["x"].shape, dev)
    s1 = torch.full(t["s0"].shape, float("nan"), dtype=torch.float32, device=dev)
    d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], y, multipass=multipass,
                                     compute=compute, backend=backend)
    if desc_hook:
        desc_hook(d)
    ids_t = None if ids is None else torch.as_tensor(np.asarray(ids, np.int32), device=dev)
    assert ctx.supported(d), ctx.last_error()
    n = ctx.scratch_size(d)
    scratch = torch.empty(max(n, 256), dtype=torch.uint8, device=dev) if n else None
    st = ctx.encode(d, t["s0"], t["x"], t["dt"], t["A"], t["B"], t["C"], y, s1, ids=ids_t,
                    scratch=scratch, stream=stream)
    assert st == abi.HELIX_OK, (st, ctx.last_error())
    torch.cuda.synchronize(dev)
    return y.cpu().numpy(), s1.cpu().numpy(), d


def widen(prob: dict, io: str) -> dict:
    """The values the kernel actually sees: bf16-rounded operands widened to
    f32 when io is bf16 (the checker must consume exactly those)."""
    if io != "bf16":
        return prob
    import torch
    out = dict(prob)
    for k in ("x", "B", "C"):
        out[k] = torch.from_numpy(np.ascontiguousarray(prob[k])).to(torch.bfloat16).float().numpy()
    return out
