"""GPU: helix_scan_encode_static, the scan for callers that cannot allocate
device memory (hosts that give an op only its inputs and outputs, so they
cannot hand helix_scan_encode a scratch buffer).  Its run scratch is a fixed
32 MiB array inside the library.

Called through the C ABI and compared with helix_scan_encode (caller-provided
scratch) on two calls in a row, for both kernel families, with many runs so
the scratch actually carries state.  This file sorts last so that a run that
stops at the first failure has already run every other test."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import helix_b200
from gpu_harness import BF16_ABS, BF16_REL, F32_ABS, F32_REL
from helpers import compare
from helix_b200 import abi

pytestmark = pytest.mark.gpu


def _tensors(seed, io, dev, L=2048, S=2, H=8, P=64, N=128, G=2):
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = dict(s0=torch.randn(S, H, P, N, generator=g) * 0.1, x=torch.randn(S, L, H, P, generator=g),
             dt=torch.randn(S, L, H, generator=g) - 4.6, A=-torch.exp(torch.rand(H, generator=g) * 2.7),
             B=torch.randn(S, L, G, N, generator=g) / N ** 0.5, C=torch.randn(S, L, G, N, generator=g) / N ** 0.5)
    t = {k: v.to(dev) for k, v in t.items()}
    for k in ("x", "B", "C"):
        t[k] = t[k].to(io)
    return t


def _static(ctx, d, t, y, s1):
    T = helix_b200._t
    return ctx.lib.helix_scan_encode_static(ctx.handle, C.c_void_p(torch.cuda.current_stream().cuda_stream),
                                            C.byref(d), T(t["s0"]), T(t["x"]), T(t["dt"]), T(t["A"]),
                                            T(t["B"]), T(t["C"]), abi.NULL_TENSOR, T(y), T(s1))


@pytest.mark.parametrize("compute", ["bf16", "f32"])
def test_static_scratch_matches_caller_scratch(ctx, cuda, compute):
    os.environ["HELIX_RUN_TOKENS"] = "256"  # 8 runs per sequence: the scratch carries state
    try:
        io = torch.bfloat16 if compute == "bf16" else torch.float32
        rel, abs_ = (BF16_REL, BF16_ABS) if compute == "bf16" else (F32_REL, F32_ABS)
        for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
            t = _tensors(seed, io, cuda)
            y_ref, s_ref = helix_b200.scan(t["x"], t["dt"], t["A"], t["B"], t["C"], t["s0"],
                                           multipass=True, compute=compute, ctx=ctx)
            y = torch.full_like(y_ref, float("nan"))
            s1 = torch.full_like(s_ref, float("nan"))
            d = helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], y, multipass=True,
                                             compute=compute)
            assert ctx.scratch_size(d) > 0
            st = _static(ctx, d, t, y, s1)
            assert st == abi.HELIX_OK, ctx.last_error()
            torch.cuda.synchronize()
            for got, want in ((y, y_ref), (s1, s_ref)):
                c = compare(got.cpu().numpy(), want.cpu().numpy(), rel, abs_)
                assert c["ok"], (compute, call, c)
    finally:
        os.environ.pop("HELIX_RUN_TOKENS", None)


def test_static_scratch_rejects_oversized(ctx, cuda):
    # 512 runs x 64 heads of 32 KiB states: far beyond the 32 MiB array.
    os.environ["HELIX_RUN_TOKENS"] = "128"
    try:
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
        assert "32" in ctx.last_error() or "bytes" in ctx.last_error()
        torch.cuda.synchronize()
        assert bool(torch.isnan(y).all()), "nothing may be enqueued on rejection"
    finally:
        os.environ.pop("HELIX_RUN_TOKENS", None)
