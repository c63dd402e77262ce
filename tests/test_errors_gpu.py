"""GPU: error conventions of the C ABI (reference include/helix/helix.h:42-49,
src/runtime/dispatch.mm:99-159): every rejection returns its status code,
records a message, and enqueues nothing (outputs stay untouched)."""
import ctypes as C

import numpy as np
import pytest
import torch

import helix_b200
from helix_b200 import abi

pytestmark = pytest.mark.gpu


def _problem(dev, L=130, S=1, H=2, P=64, N=128, G=1):
    g = torch.Generator(device="cpu").manual_seed(3)
    t = dict(s0=torch.randn(S, H, P, N, generator=g), x=torch.randn(S, L, H, P, generator=g),
             dt=torch.randn(S, L, H, generator=g) - 3, A=-torch.rand(H, generator=g) - 0.5,
             B=torch.randn(S, L, G, N, generator=g) / 11, C=torch.randn(S, L, G, N, generator=g) / 11)
    t = {k: v.to(dev) for k, v in t.items()}
    t["y"] = torch.full_like(t["x"], float("nan"))
    t["s1"] = torch.full_like(t["s0"], float("nan"))
    return t


def _desc(t, multipass=True):
    return helix_b200.desc_from_tensors(t["x"], t["dt"], t["B"], t["s0"], t["y"], multipass=multipass)


def _enc(ctx, d, t, scratch=None, **over):
    a = dict(t, **over)
    return ctx.encode(d, a["s0"], a["x"], a["dt"], a["A"], a["B"], a["C"], a["y"], a["s1"],
                      scratch=scratch)


def _untouched(t):
    torch.cuda.synchronize()
    return bool(torch.isnan(t["y"]).all()) and bool(torch.isnan(t["s1"]).all())


def test_unsupported_diagonal_a(ctx, cuda):
    t = _problem(cuda)
    d = _desc(t, multipass=False)
    d.a_form = abi.HELIX_A_DIAG_PER_CHANNEL
    assert not ctx.supported(d)
    assert "diagonal" in ctx.last_error()
    assert _enc(ctx, d, t) == abi.HELIX_ERR_UNSUPPORTED_SHAPE
    assert ctx.backend_desc(d).startswith("declined")
    assert _untouched(t)


def test_unsupported_shapes(ctx, cuda):
    t = _problem(cuda)
    for hook in (lambda d: setattr(d, "n_group", 3), lambda d: setattr(d, "d_state", 12),
                 lambda d: setattr(d, "chunk", 32), lambda d: setattr(d, "io_dtype", abi.HELIX_F16),
                 lambda d: d.s_b.__setitem__(2, 2), lambda d: setattr(d, "n_tok", 0)):
        d = _desc(t, multipass=False)
        hook(d)
        assert not ctx.supported(d)
        assert _enc(ctx, d, t) == abi.HELIX_ERR_UNSUPPORTED_SHAPE
    assert _untouched(t)


def test_null_tensor(ctx, cuda):
    t = _problem(cuda)
    d = _desc(t, multipass=False)
    assert _enc(ctx, d, t, x=None) == abi.HELIX_ERR_INVALID_ARG
    assert _untouched(t)


def test_missing_and_small_scratch(ctx, cuda):
    t = _problem(cuda, L=1024, H=4)
    d = _desc(t, multipass=True)
    need = ctx.scratch_size(d)
    assert need > 0
    assert _enc(ctx, d, t) == abi.HELIX_ERR_SCRATCH_TOO_SMALL
    # an exact-size cudaMalloc that is too small by one page
    rt = C.CDLL("libcudart.so.12")
    ptr = C.c_void_p()
    assert rt.cudaMalloc(C.byref(ptr), C.c_size_t(need - 4096)) == 0
    try:
        st = ctx.lib.helix_scan_encode(ctx.handle, None, C.byref(d), *[helix_b200._t(t[k]) for k in
                                       ("s0", "x", "dt", "A", "B", "C")], abi.NULL_TENSOR,
                                       helix_b200._t(t["y"]), helix_b200._t(t["s1"]), abi.Tensor(ptr, 0))
        assert st == abi.HELIX_ERR_SCRATCH_TOO_SMALL
        # misaligned scratch
        st = ctx.lib.helix_scan_encode(ctx.handle, None, C.byref(d), *[helix_b200._t(t[k]) for k in
                                       ("s0", "x", "dt", "A", "B", "C")], abi.NULL_TENSOR,
                                       helix_b200._t(t["y"]), helix_b200._t(t["s1"]), abi.Tensor(ptr, 16))
        assert st == abi.HELIX_ERR_INVALID_ARG
    finally:
        torch.cuda.synchronize()
        rt.cudaFree(ptr)
    assert _untouched(t)


def test_overlapping_states(ctx, cuda):
    t = _problem(cuda)
    d = _desc(t, multipass=False)
    assert _enc(ctx, d, t, s1=t["s0"]) == abi.HELIX_ERR_INVALID_ARG
    assert "overlap" in ctx.last_error()


def test_encode_into_same_as_encode(ctx, cuda):
    t = _problem(cuda)
    d = _desc(t, multipass=False)
    assert _enc(ctx, d, t) == abi.HELIX_OK
    torch.cuda.synchronize()
    y1 = t["y"].clone()
    t["y"].fill_(float("nan"))
    st = ctx.encode(d, t["s0"], t["x"], t["dt"], t["A"], t["B"], t["C"], t["y"], t["s1"], into=True)
    assert st == abi.HELIX_OK
    torch.cuda.synchronize()
    assert torch.equal(y1, t["y"])


def test_ctx_on_explicit_device_and_descriptions(cuda):
    c = helix_b200.Context(0)
    t = _problem(cuda)
    d = _desc(t)
    assert "fp32" in c.backend_desc(d)
    d.compute_dtype = abi.HELIX_BF16
    c.close()


def test_bad_device_ordinal():
    with pytest.raises(helix_b200.HelixError) as e:
        helix_b200.Context(10_000)
    assert e.value.status == abi.HELIX_ERR_NO_DEVICE
