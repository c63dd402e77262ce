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


def test_unsupported_a_form(ctx, cuda):
    t = _problem(cuda)
    d = _desc(t, multipass=False)
    d.a_form = 7  # neither helix_a_form value
    assert not ctx.supported(d)
    assert "a_form" in ctx.last_error()
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


def _fault(ctx):
    code = C.c_uint32(0)
    assert ctx.lib.helix_device_fault(ctx.handle, C.byref(code)) == abi.HELIX_OK
    return code.value


@pytest.mark.parametrize("compute,multipass", [("f32", False), ("f32", True), ("bf16", False), ("bf16", True)])
def test_ids_row_overlapping_s1(ctx, cuda, compute, multipass):
    """ids may select any row of s0, beyond the n_seq rows the host can check.
    A selected row that overlaps the s1 rows being written is not read: that
    sequence comes out NaN and the fault word records code 5; a row clear of
    s1 in the same allocation runs normally."""
    t = _problem(cuda, L=300, H=2)
    S, H, P, N = t["s0"].shape
    buf = torch.randn(4, S, H, P, N, device=cuda) * 0.1  # rows 0..3 of one allocation
    s1 = buf[2]
    io = torch.bfloat16 if compute == "bf16" else torch.float32
    x, B, Cm = t["x"].to(io), t["B"].to(io), t["C"].to(io)
    d = helix_b200.desc_from_tensors(x, t["dt"], B, buf[0], t["y"], multipass=multipass, compute=compute)
    n = ctx.scratch_size(d)
    scratch = torch.empty(max(n, 256), dtype=torch.uint8, device=cuda) if n else None
    _fault(ctx)  # clear
    for row, bad in ((2, True), (3, False)):
        ids = torch.tensor([row], dtype=torch.int32, device=cuda)
        t["y"].fill_(0.0)
        s1.fill_(0.0)
        st = ctx.encode(d, buf[0], x, t["dt"], t["A"], B, Cm, t["y"], s1, ids=ids, scratch=scratch)
        assert st == abi.HELIX_OK, ctx.last_error()
        torch.cuda.synchronize()
        code = _fault(ctx)
        if bad:
            assert code == 5, code
            assert bool(torch.isnan(t["y"]).all()) and bool(torch.isnan(s1).all())
        else:
            assert code == 0, code
            assert bool(torch.isfinite(t["y"]).all()) and bool(torch.isfinite(s1).all())


def test_carry_combine_ids_row_overlapping_carry(ctx, cuda):
    S, H, P, N = 1, 2, 64, 128
    buf = torch.randn(4, S, H, P, N, device=cuda)
    x = torch.empty(S, 128, H, P, device=cuda)
    dt = torch.empty(S, 128, H, device=cuda)
    Bm = torch.empty(S, 128, 1, N, device=cuda)
    d = helix_b200.desc_from_tensors(x, dt, Bm, buf[0], multipass=True)
    _fault(ctx)
    for row, bad in ((1, True), (3, False)):
        ids = torch.tensor([row], dtype=torch.int32, device=cuda)
        carry = buf[1]
        st = ctx.encode_carry_combine(d, buf[0], buf[:0], torch.empty(0, device=cuda), 0, carry, ids=ids)
        assert st == abi.HELIX_OK, ctx.last_error()
        torch.cuda.synchronize()
        assert _fault(ctx) == (5 if bad else 0)
        assert bool(torch.isnan(carry).all()) == bad


def test_error_strings_per_thread_and_freed_with_context(cuda):
    import threading
    t = _problem(cuda)
    a = helix_b200.Context(0)
    d = _desc(t, multipass=False)
    d.a_form = 7
    assert not a.supported(d)
    assert "a_form" in a.last_error()
    seen = {}
    th = threading.Thread(target=lambda: seen.setdefault("other", a.last_error()))
    th.start()
    th.join()
    assert seen["other"] == ""  # another thread has no error on this context
    a.close()
    for _ in range(8):  # later contexts start clean, wherever they are allocated
        b = helix_b200.Context(0)
        assert b.last_error() == ""
        b.close()


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


def test_bounded_wait_expires_and_the_gpu_recovers(ctx, oracle):
    """The tensor-core output kernel's waits are bounded.  With the test hook
    HELIX_TEST_STALL_CYCLES each of its CTAs first waits, with that short
    budget, on a barrier nothing arrives on: the wait must run out, the
    kernel must return (the stream synchronises), the fault word must read
    code 6 and the tiles it owns stay unwritten.  The next scan on the same
    context, without the hook, must be correct and record no fault."""
    import os

    from gpu_harness import BF16_ABS, BF16_REL, run, widen
    from helpers import compare
    shape = (512, 1, 4, 64, 128, 2)
    prob = widen(oracle.harness_problem(*shape, 4242, True), "bf16")
    d = oracle.desc_init(*shape)
    y_ref, _ = oracle.scan(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")])
    _fault(ctx)  # clear
    os.environ["HELIX_TEST_STALL_CYCLES"] = "200000"
    try:
        y, s1, _ = run(ctx, prob, multipass=True, io="bf16", compute="bf16")
    finally:
        os.environ.pop("HELIX_TEST_STALL_CYCLES", None)
    assert _fault(ctx) == 6
    assert np.isnan(y).all() and np.isnan(s1).all()
    y, s1, _ = run(ctx, prob, multipass=True, io="bf16", compute="bf16")
    assert _fault(ctx) == 0
    c = compare(y, y_ref, BF16_REL, BF16_ABS)
    assert c["ok"], c
