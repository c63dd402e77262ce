"""GPU: scans captured into a CUDA graph and replayed with new inputs.

ggml-cuda captures its ops into CUDA graphs, and a serving loop replays
graphs rather than re-encoding; helix_scan_encode must therefore enqueue
nothing a stream capture rejects (no host synchronisation, no allocation, no
blocking copy) and its kernel-to-kernel programmatic launches must survive
capture.  Each family is captured once and replayed on two fresh problems
copied into the captured buffers, against the fp64 oracle at that family's
bound; HELIX_RUN_TOKENS=128 at capture time puts run boundaries in, so the
state and carry kernels are part of the graph."""
import os

import numpy as np
import pytest

from gpu_harness import BF16_ABS, BF16_REL, BF16_RL2, F32_ABS, F32_REL, F32_RL2, X3_ABS, X3_REL, X3_RL2, widen
from helpers import compare
from helix_b200 import abi
from oracle.oracle import diag_desc

pytestmark = pytest.mark.gpu

SHAPE = (600, 2, 8, 64, 128, 2)  # L, S, H, P, N, G
BF16 = (BF16_REL, BF16_ABS, BF16_RL2)
S1_BF16 = (2e-5, 2e-6, 1e-4)  # the bf16 family's state stays fp32 (its parity suite's s1 bound)
X3 = (X3_REL, X3_ABS, X3_RL2)
F32 = (F32_REL, F32_ABS, F32_RL2)
# name, x/B/C storage, compute, backend, diagonal A, bound of y, bound of s1
FAMILIES = [
    ("bf16", "bf16", "bf16", abi.HELIX_BACKEND_AUTO, False, BF16, S1_BF16),
    ("bf16_f32_stored", "f32", "bf16", abi.HELIX_BACKEND_AUTO, False, BF16, S1_BF16),
    ("fp32_tensor_core", "f32", "f32", abi.HELIX_BACKEND_AUTO, False, X3, X3),
    ("exact_fp32", "f32", "f32", abi.HELIX_BACKEND_REF, False, F32, F32),
    ("diagonal_a", "f32", "f32", abi.HELIX_BACKEND_AUTO, True, X3, X3),
]


@pytest.fixture
def runs128():
    old = os.environ.get("HELIX_RUN_TOKENS")
    os.environ["HELIX_RUN_TOKENS"] = "128"
    yield
    if old is None:
        os.environ.pop("HELIX_RUN_TOKENS", None)
    else:
        os.environ["HELIX_RUN_TOKENS"] = old


def _problem(oracle, seed, diag):
    make = oracle.harness_problem_diag if diag else oracle.harness_problem
    prob = make(*SHAPE, seed, True)
    prob["s0"] = np.random.default_rng(seed).normal(0, 0.1, prob["s0"].shape).astype(np.float32)
    return prob


@pytest.mark.parametrize("fam", FAMILIES, ids=[f[0] for f in FAMILIES])
def test_captured_scan_replays(ctx, oracle, runs128, fam):
    import torch
    import helix_b200
    name, io, compute, backend, diag, y_bound, s1_bound = fam
    dev = torch.device("cuda:0")
    io_t = torch.bfloat16 if io == "bf16" else torch.float32
    first = _problem(oracle, 11, diag)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in first.items()}
    for k in ("x", "B", "C"):
        t[k] = t[k].to(io_t)
    y = torch.full(t["x"].shape, float("nan"), dtype=torch.float32, device=dev)
    s1 = torch.full(t["s0"].shape, float("nan"), dtype=torch.float32, device=dev)
    d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], y, multipass=True, compute=compute,
                                     backend=backend, A=t["A"])
    assert ctx.supported(d), ctx.last_error()
    scratch = torch.empty(max(ctx.scratch_size(d), 256), dtype=torch.uint8, device=dev)
    args = (d, t["s0"], t["x"], t["dt"], t["A"], t["B"], t["C"], y, s1)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # one eager run before capture
        assert ctx.encode(*args, scratch=scratch) == abi.HELIX_OK
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st = ctx.encode(*args, scratch=scratch)
    assert st == abi.HELIX_OK, ctx.last_error()

    for seed in (12, 13):
        prob = _problem(oracle, seed, diag)
        for k in ("s0", "x", "dt", "A", "B", "C"):
            t[k].copy_(torch.from_numpy(np.ascontiguousarray(prob[k])).to(dev).to(t[k].dtype))
        y.fill_(float("nan"))
        s1.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize(dev)
        seen = widen(prob, "bf16" if compute == "bf16" else io)  # what the kernels read
        od = oracle.desc_init(*SHAPE)
        if diag:
            diag_desc(od)
        y_ref, s_ref = oracle.scan(od, *[seen[k] for k in ("s0", "x", "dt", "A", "B", "C")])
        for got, want, what, (rel, ab, rl2) in ((y, y_ref, "y", y_bound), (s1, s_ref, "s1", s1_bound)):
            c = compare(got.cpu().numpy(), want, rel, ab)
            assert c["ok"] and c["rel_l2"] <= rl2, (name, seed, what, c)
    del g
