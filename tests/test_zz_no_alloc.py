"""GPU: helix_scan_encode_static, the scan for callers that cannot allocate
device memory (hosts that give an op only its inputs and outputs, so they
cannot hand helix_scan_encode a scratch buffer).  Its run scratch is a fixed
32 MiB array inside the library.

Called through the C ABI and checked on consecutive calls against both
helix_scan_encode (caller scratch, NaN-filled before each call) and the fp64
oracle on the same inputs, within the bounds the parity suites use:
  * two calls in a row of one shape, both kernel families;
  * a larger call with a different run plan first, then a smaller, ragged one
    (so the second call reads an array the first one laid out differently),
    with one chunk of extreme decay routing tiles of the tensor-core family
    through the general path (which reads the run spans and tile flags from
    the shared array);
  * diagonal A (the recurrence kernels' run states and dt sums in the array);
  * in a fresh process, the array is reserved by the first call and not
    before (lazy module loading).
This file sorts last so that a run that stops at the first failure has
already run every other test; each case sets up what it needs, so the file
also passes on its own."""
import ctypes as C
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import helix_b200
from gpu_harness import BF16_ABS, BF16_REL, BF16_RL2, X3_ABS, X3_REL, X3_RL2, widen
from helpers import compare
from helix_b200 import abi

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
S1_BF16 = (2e-5, 2e-6, 1e-4)  # the carried state keeps fp32-like bounds on the bf16 path


def _problem(oracle, seed, L, S, H, P, N, G, hot_chunk=None):
    """The reference harness's inputs (the regime the parity bounds are
    calibrated on); hot_chunk=(t0, h) gives head h one 128-token chunk with
    softplus(dt) ~ 6 per token (hundreds of nats of decay)."""
    prob = oracle.harness_problem(L, S, H, P, N, G, seed, True)
    if hot_chunk is not None:
        t0, h = hot_chunk
        prob["dt"][:, t0:t0 + 128, h] = 6.0
    return prob


def _torch(prob, io, dev):
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
    for k in ("x", "B", "C"):
        t[k] = t[k].to(io)
    return t


def _static(ctx, d, t, y, s1):
    T = helix_b200._t
    return ctx.lib.helix_scan_encode_static(ctx.handle, C.c_void_p(torch.cuda.current_stream().cuda_stream),
                                            C.byref(d), T(t["s0"]), T(t["x"]), T(t["dt"]), T(t["A"]),
                                            T(t["B"]), T(t["C"]), abi.NULL_TENSOR, T(y), T(s1))


def _check_call(ctx, oracle, prob, shape, compute, tag):
    L, S, H, P, N, G = shape
    dev = torch.device("cuda:0")
    io = torch.bfloat16 if compute == "bf16" else torch.float32
    t = _torch(prob, io, dev)
    d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], multipass=True, compute=compute)
    assert ctx.supported(d), ctx.last_error()
    need = ctx.scratch_size(d)
    assert 0 < need <= (32 << 20)
    # the existing entry point, its caller scratch full of NaN
    scratch = torch.full((need // 4 + 64,), float("nan"), device=dev)
    y_enc = torch.full((S, L, H, P), float("nan"), device=dev)
    s_enc = torch.full((S, H, P, N), float("nan"), device=dev)
    assert ctx.encode(d, t["s0"], t["x"], t["dt"], t["A"], t["B"], t["C"], y_enc, s_enc,
                      scratch=scratch) == abi.HELIX_OK, ctx.last_error()
    y = torch.full_like(y_enc, float("nan"))
    s1 = torch.full_like(s_enc, float("nan"))
    assert _static(ctx, d, t, y, s1) == abi.HELIX_OK, ctx.last_error()
    torch.cuda.synchronize()
    w = widen(prob, "bf16" if compute == "bf16" else "f32")
    od = oracle.desc_init(L, S, H, P, N, G)
    y_ref, s_ref = oracle.scan(od, *[w[k] for k in ("s0", "x", "dt", "A", "B", "C")])
    if compute == "bf16":
        yb, sb = (BF16_REL, BF16_ABS, BF16_RL2), S1_BF16
    else:  # compute F32 on F32-stored inputs: the fp32-class tensor-core family
        yb = sb = (X3_REL, X3_ABS, X3_RL2)
    got = dict(y=y.cpu().numpy(), s1=s1.cpu().numpy())
    enc = dict(y=y_enc.cpu().numpy(), s1=s_enc.cpu().numpy())
    for name, want, (rel, abs_, rl2) in (("y", y_ref, yb), ("s1", s_ref, sb)):
        c = compare(got[name], want, rel, abs_)
        assert c["ok"] and c["rel_l2"] <= rl2, (tag, name, "vs oracle", c)
        c = compare(got[name], enc[name], rel, abs_)
        assert c["ok"], (tag, name, "vs helix_scan_encode", c)


@pytest.fixture
def env():
    saved = {k: os.environ.get(k) for k in ("HELIX_RUN_TOKENS", "HELIX_TC_GENERAL")}

    def set_(k, v):
        os.environ[k] = v
    yield set_
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


@pytest.mark.parametrize("compute", ["bf16", "f32"])
def test_static_two_calls_in_a_row(ctx, oracle, env, compute):
    env("HELIX_RUN_TOKENS", "256")  # 8 runs per sequence: the array carries run states
    shape = (2048, 2, 8, 64, 128, 2)
    for call, seed in enumerate((11, 12)):
        _check_call(ctx, oracle, _problem(oracle, seed, *shape), shape, compute, f"{compute} call {call}")


@pytest.mark.parametrize("compute", ["bf16", "f32"])
def test_static_larger_plan_then_smaller(ctx, oracle, env, compute):
    # first call: 4096 tokens in 16 runs of 256, 8 heads; a hot chunk in head 3
    env("HELIX_RUN_TOKENS", "256")
    big = (4096, 1, 8, 64, 128, 2)
    _check_call(ctx, oracle, _problem(oracle, 21, *big, hot_chunk=(1024 + 128, 3)), big, compute,
                f"{compute} big")
    # second call: ragged 1000 tokens, wide heads, one group, the planner's own
    # run cut; a hot chunk in head 1 of the last span
    os.environ.pop("HELIX_RUN_TOKENS", None)
    small = (1000, 2, 4, 128, 128, 1)
    _check_call(ctx, oracle, _problem(oracle, 22, *small, hot_chunk=(768, 1)), small, compute,
                f"{compute} small")


def test_static_general_path_forced(ctx, oracle, env):
    env("HELIX_RUN_TOKENS", "256")
    env("HELIX_TC_GENERAL", "1")
    shape = (1536, 1, 4, 64, 128, 2)
    _check_call(ctx, oracle, _problem(oracle, 31, *shape), shape, "bf16", "bf16 forced general")


def test_static_diagonal_a(ctx, oracle, env):
    """Diagonal A through the static array: its run states and dt sums."""
    from oracle.oracle import diag_desc
    env("HELIX_RUN_TOKENS", "256")
    shape = (1000, 2, 8, 64, 64, 2)
    L, S, H, P, N, G = shape
    dev = torch.device("cuda:0")
    prob = oracle.harness_problem_diag(*shape, 41, True)
    t = _torch(prob, torch.float32, dev)
    d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], multipass=True, A=t["A"])
    assert d.a_form == abi.HELIX_A_DIAG_PER_CHANNEL and 0 < ctx.scratch_size(d) <= (32 << 20)
    for call in range(2):
        y = torch.full((S, L, H, P), float("nan"), device=dev)
        s1 = torch.full((S, H, P, N), float("nan"), device=dev)
        assert _static(ctx, d, t, y, s1) == abi.HELIX_OK, ctx.last_error()
        torch.cuda.synchronize()
        y_ref, s_ref = oracle.scan(diag_desc(oracle.desc_init(*shape)),
                                   *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")])
        for name, got, want in (("y", y, y_ref), ("s1", s1, s_ref)):
            c = compare(got.cpu().numpy(), want, X3_REL, X3_ABS)
            assert c["ok"] and c["rel_l2"] <= X3_RL2, ("diag", call, name, c)


def test_static_scratch_rejects_oversized(ctx, cuda, env):
    # 512 runs x 64 heads of 32 KiB states: far beyond the 32 MiB array.
    env("HELIX_RUN_TOKENS", "128")
    L, H, P, N, G = 65536, 64, 64, 128, 8
    bf = dict(dtype=torch.bfloat16, device=cuda)
    t = dict(s0=torch.zeros(1, H, P, N, device=cuda), x=torch.empty(1, L, H, P, **bf),
             dt=torch.empty(1, L, H, device=cuda), A=torch.empty(H, device=cuda),
             B=torch.empty(1, L, G, N, **bf), C=torch.empty(1, L, G, N, **bf))
    y = torch.full(t["x"].shape, float("nan"), device=cuda)
    s1 = torch.full_like(t["s0"], float("nan"))
    d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], y, multipass=True)
    assert ctx.scratch_size(d) > (32 << 20)
    assert _static(ctx, d, t, y, s1) == abi.HELIX_ERR_SCRATCH_TOO_SMALL
    assert "bytes" in ctx.last_error()
    torch.cuda.synchronize()
    assert bool(torch.isnan(y).all()), "nothing may be enqueued on rejection"


_FRESH = r"""
import ctypes as C, json, sys
sys.path.insert(0, sys.argv[1])
import torch
import helix_b200
from helix_b200 import abi
rt = C.CDLL("libcudart.so.12")
def free():
    f, t = C.c_size_t(), C.c_size_t()
    assert rt.cudaMemGetInfo(C.byref(f), C.byref(t)) == 0
    return f.value
ctx = helix_b200.Context(0)
dev = torch.device("cuda:0")
g = torch.Generator(device="cpu").manual_seed(5)
L, H, P, N, G = 512, 2, 64, 128, 1
t = dict(s0=torch.zeros(1, H, P, N), x=torch.randn(1, L, H, P, generator=g),
         dt=torch.randn(1, L, H, generator=g) - 4.6, A=-torch.rand(H, generator=g) - 1,
         B=torch.randn(1, L, G, N, generator=g) / 11, C=torch.randn(1, L, G, N, generator=g) / 11)
t = {k: v.to(dev) for k, v in t.items()}
y = torch.empty_like(t["x"]); s1 = torch.empty_like(t["s0"])
d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], y, multipass=True)
T = helix_b200._t
def call():
    st = ctx.lib.helix_scan_encode_static(ctx.handle, None, C.byref(d), T(t["s0"]), T(t["x"]), T(t["dt"]),
                                          T(t["A"]), T(t["B"]), T(t["C"]), abi.NULL_TENSOR, T(y), T(s1))
    torch.cuda.synchronize()
    return st
# everything but the static array loaded: an ordinary scan first
assert ctx.encode(d, t["s0"], t["x"], t["dt"], t["A"], t["B"], t["C"], y, s1,
                  scratch=torch.empty(max(ctx.scratch_size(d), 256), dtype=torch.uint8, device=dev)) == 0
torch.cuda.synchronize()
f0 = free(); st1 = call(); f1 = free(); st2 = call(); f2 = free()
print(json.dumps(dict(st1=st1, st2=st2, first=f0 - f1, second=f1 - f2)))
"""


def test_static_array_reserved_by_first_call(cuda):
    env = dict(os.environ, CUDA_MODULE_LOADING="LAZY")
    r = subprocess.run([sys.executable, "-c", _FRESH, str(ROOT)], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["st1"] == abi.HELIX_OK and out["st2"] == abi.HELIX_OK, out
    assert out["first"] >= (30 << 20), out     # the 32 MiB array arrives with the first call
    assert abs(out["second"]) < (8 << 20), out  # and nothing more with the next
