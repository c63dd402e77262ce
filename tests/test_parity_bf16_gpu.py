"""GPU parity of the tcgen05 kernels (x, B, C stored bf16; bf16 GEMM operands,
fp32 accumulators and fp32 carried state) against the fp64 oracle run on the
same bf16-rounded inputs, through the C ABI.

Bounds: y is held to the reference's calibrated bf16 per-element bound
(reference tests/test_metal_parity.mm:35-38, rel 1.5e-2 / abs 3e-3) and to the
north star's 2e-2 relative L2.  The carried state is held to a bound 4x the
fp32 one: the state update multiplies exact bf16 B by dt*decay*x split into a
bf16 hi+lo pair (~16 mantissa bits), so the carry never passes through a
single bf16 rounding (the reference's bf16 path keeps its carry fp32 too,
test_metal_parity.mm:214-218)."""
import os
from pathlib import Path

import numpy as np
import pytest

from gpu_harness import BF16_ABS, BF16_REL, BF16_RL2, record, run, widen
from helpers import compare
from helix_b200 import abi

pytestmark = pytest.mark.gpu

S1_REL, S1_ABS, S1_RL2 = 2e-5, 2e-6, 1e-4

SHAPES = [  # reference tests/test_metal_parity.mm:77-104 (all 22 rows)
    (1, 1, 2, 64, 128, 1), (7, 1, 2, 64, 128, 1), (63, 1, 2, 64, 128, 1),
    (64, 1, 2, 64, 128, 1), (65, 1, 2, 64, 128, 1), (127, 1, 2, 64, 128, 1),
    (128, 1, 2, 64, 128, 1), (129, 1, 2, 64, 128, 1), (96, 1, 4, 64, 128, 1),
    (160, 1, 4, 64, 128, 1), (300, 1, 8, 64, 128, 2), (256, 1, 4, 64, 64, 1),
    (256, 1, 4, 128, 128, 1), (256, 1, 4, 128, 256, 1), (256, 1, 4, 64, 256, 1),
    (300, 1, 4, 128, 256, 1), (256, 1, 8, 128, 256, 2), (256, 1, 4, 192, 128, 1),
    (256, 1, 8, 128, 128, 8), (256, 4, 4, 64, 128, 1),
    (1024, 1, 2, 64, 128, 1), (2048, 1, 8, 64, 128, 2), (200, 1, 2, 72, 128, 1),
    # output tiles pair two slabs of a group: an odd slab count leaves the
    # last pair half empty; many pairs make the planner give each output CTA
    # a span of several runs
    (192, 1, 3, 64, 128, 1), (256, 2, 8, 64, 128, 8), (1024, 1, 128, 64, 128, 1),
]
MODES = [("1pass", False, None), ("multipass", True, None), ("multipass/runs128", True, "128")]


@pytest.fixture
def run_tokens():
    old = os.environ.get("HELIX_RUN_TOKENS")

    def set_(v):
        if v is None:
            os.environ.pop("HELIX_RUN_TOKENS", None)
        else:
            os.environ["HELIX_RUN_TOKENS"] = v
    yield set_
    set_(old)


@pytest.fixture
def tc_general():
    """HELIX_TC_GENERAL=1 sends every output CTA down the general path (the
    default picks the fast path per run when no chunk decays by more than ~60
    nats; the SHORT harness regime has heads on both sides of that line)."""
    old = os.environ.get("HELIX_TC_GENERAL")

    def set_(on):
        if on:
            os.environ["HELIX_TC_GENERAL"] = "1"
        else:
            os.environ.pop("HELIX_TC_GENERAL", None)
    yield set_
    set_(old)


def check_bf16(tag, y, s1, y_ref, s_ref):
    cy = compare(y, y_ref, BF16_REL, BF16_ABS)
    cs = compare(s1, s_ref, S1_REL, S1_ABS)
    record(tag, y_ratio=cy["ratio"], y_rl2=cy["rel_l2"], s_ratio=cs["ratio"], s_rl2=cs["rel_l2"])
    assert cy["ok"] and cy["rel_l2"] <= BF16_RL2, (tag, "y", cy)
    assert cs["ok"] and cs["rel_l2"] <= S1_RL2, (tag, "s1", cs)


def _oracle(oracle, prob, shape, ids=None, threads=1):
    L, S, H, P, N, G = shape
    d = oracle.desc_init(L, S, H, P, N, G)
    args = [prob[k] for k in ("s0", "x", "dt", "A", "B", "C")]
    if threads > 1:
        return oracle.scan_mt(d, *args, ids=ids, threads=threads)
    return oracle.scan(d, *args, ids=ids)


@pytest.mark.parametrize("path", ["auto", "general"])
@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
@pytest.mark.parametrize("mode", MODES, ids=[m[0] for m in MODES])
@pytest.mark.parametrize("shape", SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in SHAPES])
def test_parity_bf16(ctx, oracle, run_tokens, tc_general, shape, mode, long_mem, path):
    name, multipass, rt = mode
    prob = widen(oracle.harness_problem(*shape, 4242, long_mem), "bf16")
    y_ref, s_ref = _oracle(oracle, prob, shape)
    run_tokens(rt)
    tc_general(path == "general")
    y, s1, d = run(ctx, prob, multipass=multipass, io="bf16", compute="bf16")
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_MPP
    assert "tcgen05" in ctx.backend_desc(d)
    check_bf16(f"bf16 {path} {name} {'long' if long_mem else 'short'} {shape}", y, s1, y_ref, s_ref)


def test_ids_and_batched_bf16(ctx, oracle, run_tokens):
    shape = (300, 3, 4, 64, 128, 2)
    prob = widen(oracle.harness_problem(*shape, 777, True), "bf16")
    ids = np.array([2, 0, 1], np.int32)
    y_ref, s_ref = _oracle(oracle, prob, shape, ids=ids)
    run_tokens("128")
    y, s1, _ = run(ctx, prob, multipass=True, io="bf16", compute="bf16", ids=ids)
    check_bf16("bf16 ids", y, s1, y_ref, s_ref)


def _y_padded_head(shape, dev):
    """y inside a buffer whose head rows are P + 1 floats apart."""
    import torch
    S, L, H, P = shape
    return torch.full((S, L, H, P + 1), float("nan"), dtype=torch.float32, device=dev)[..., :P]


def _y_offset(shape, dev):
    """Dense y starting 4 bytes past a 16-byte boundary."""
    import torch
    n = int(np.prod(shape))
    return torch.full((n + 1,), float("nan"), dtype=torch.float32, device=dev)[1:].view(shape)


@pytest.mark.parametrize("y_view", [_y_padded_head, _y_offset], ids=["padded_head", "offset"])
def test_strided_y_bf16(ctx, oracle, y_view):
    """y written through a view: a head stride that is not a multiple of
    four floats, and a base 4 bytes past a 16-byte boundary."""
    shape = (300, 2, 4, 64, 128, 2)
    prob = widen(oracle.harness_problem(*shape, 99, True), "bf16")
    y_ref, s_ref = _oracle(oracle, prob, shape)
    y, s1, d = run(ctx, prob, multipass=True, io="bf16", compute="bf16", y_view=y_view)
    assert "tcgen05" in ctx.backend_desc(d)
    check_bf16(f"bf16 strided y {y_view.__name__}", y, s1, y_ref, s_ref)


@pytest.mark.parametrize("span", [1, 3], ids=["inner_span", "last_span"])
def test_fast_general_decision_from_state_pass(ctx, oracle, run_tokens, span):
    """With a state pass, the output kernels take the fast/general decision
    from the decay spans the state pass records per run: for the runs it
    reduces, and for the last output span (which it does not reduce) from an
    extra measurement.  One chunk of head 0 decays by hundreds of nats inside
    the given span; the fast path's rescaling factors would overflow there,
    so only a tile sent down the general path gives finite, correct output."""
    shape = (2048, 1, 4, 64, 128, 2)
    prob = oracle.harness_problem(*shape, 4242, True)
    t0 = 512 * span + 128
    prob["dt"][:, t0:t0 + 128, 0] = 6.0  # softplus(6) ~ 6 per token
    prob = widen(prob, "bf16")
    y_ref, s_ref = _oracle(oracle, prob, shape)
    run_tokens("512")  # four output spans of one run each: a state pass over runs 0..2
    y, s1, d = run(ctx, prob, multipass=True, io="bf16", compute="bf16")
    assert "tcgen05" in ctx.backend_desc(d)
    assert np.isfinite(y).all() and np.isfinite(s1).all()
    check_bf16(f"bf16 decision from state pass span {span}", y, s1, y_ref, s_ref)


def test_c3_full_size_bf16(ctx, oracle):
    """BASELINE config 3 at full size on the BASELINE distributions."""
    from helix_b200.synth import Shape, make_inputs, to_numpy_f32
    sh = Shape.of("c3")
    t = make_inputs(sh, seed=1234, s0_std=0.1)
    prob = {k: to_numpy_f32(t[k]) for k in ("s0", "x", "dt", "A", "B", "C")}
    y_ref, s_ref = _oracle(oracle, prob, (sh.L, sh.S, sh.H, sh.P, sh.N, sh.G), threads=os.cpu_count() or 1)
    y, s1, _ = run(ctx, prob, multipass=True, io="bf16", compute="bf16")
    check_bf16("bf16 c3", y, s1, y_ref, s_ref)


def test_no_device_fault_recorded(ctx):
    import ctypes as C
    code = C.c_uint32(123)
    assert ctx.lib.helix_device_fault(ctx.handle, C.byref(code)) == abi.HELIX_OK
    assert code.value == 0


# F32-stored x, B, C on the tensor-core family: a cast kernel makes dense bf16
# copies in the scratch first (the reference's bf16 Pass C casts B and C the
# same way, src/kernels/helix_cast.metal:19-46).  Shapes cover d_state 64, 128
# and 256, ragged L, a head_dim that is not a multiple of 64 and several runs.
F32IO_SHAPES = [(129, 1, 2, 64, 128, 1), (300, 1, 8, 64, 128, 2), (256, 1, 4, 64, 64, 1),
                (300, 1, 4, 128, 256, 1), (256, 1, 8, 128, 256, 2), (200, 1, 2, 72, 128, 1),
                (1000, 2, 4, 192, 128, 1), (2048, 1, 8, 64, 128, 2)]


@pytest.mark.parametrize("rt", [None, "128"], ids=["planned", "runs128"])
@pytest.mark.parametrize("shape", F32IO_SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in F32IO_SHAPES])
def test_parity_bf16_f32_io(ctx, oracle, run_tokens, shape, rt):
    prob = oracle.harness_problem(*shape, 4242, True)
    # the kernels see x, B, C rounded to bf16 once: check their arithmetic on
    # exactly those values
    y_ref, s_ref = _oracle(oracle, widen(prob, "bf16"), shape)
    run_tokens(rt)
    y, s1, d = run(ctx, prob, multipass=True, io="f32", compute="bf16")
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_MPP
    assert "tcgen05" in ctx.backend_desc(d)
    check_bf16(f"bf16 f32-io {rt} {shape}", y, s1, y_ref, s_ref)


def test_f32_io_single_pass_takes_fp32_family(ctx, oracle):
    """Single pass has no scratch for the bf16 copies: F32-stored inputs with
    compute BF16 run on the exact fp32 family (as the reference's bf16 Pass C
    needs multipass)."""
    shape = (300, 1, 4, 64, 128, 1)
    prob = oracle.harness_problem(*shape, 4242, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    y, s1, d = run(ctx, prob, multipass=False, io="f32", compute="bf16")
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_REF
    c = compare(y, y_ref, 5e-6, 5e-7)
    assert c["ok"], c


def test_f32_io_strided_x(ctx, oracle):
    """x read through a view (head rows P + 3 floats apart, channels two
    floats apart): the cast kernel's strided path."""
    import torch
    shape = (300, 2, 4, 64, 128, 2)
    prob = oracle.harness_problem(*shape, 7, True)
    y_ref, s_ref = _oracle(oracle, widen(prob, "bf16"), shape)

    L, S, H, P, N, G = shape
    dev = torch.device("cuda:0")
    big = torch.full((S, L, H, 2 * P + 3), float("nan"), device=dev)
    x = big[..., : 2 * P : 2]
    x.copy_(torch.from_numpy(prob["x"]).to(dev))
    t = {k: torch.from_numpy(np.ascontiguousarray(prob[k])).to(dev) for k in ("s0", "dt", "A", "B", "C")}
    import helix_b200
    y = torch.full((S, L, H, P), float("nan"), device=dev)
    s1 = torch.full_like(t["s0"], float("nan"))
    d = helix_b200.desc_from_tensors(x, t["dt"], t["B"], t["s0"], y, multipass=True, compute="bf16")
    assert ctx.supported(d), ctx.last_error()
    scratch = torch.empty(ctx.scratch_size(d), dtype=torch.uint8, device=dev)
    assert ctx.encode(d, t["s0"], x, t["dt"], t["A"], t["B"], t["C"], y, s1, scratch=scratch) == abi.HELIX_OK
    torch.cuda.synchronize()
    check_bf16("bf16 f32-io strided x", y.cpu().numpy(), s1.cpu().numpy(), y_ref, s_ref)


GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_bf16(ctx, oracle, run_tokens, path):
    """The committed outputs of the reference's own fp64 oracle, on its
    F32-stored inputs, through the tensor-core family (inputs rounded to bf16
    by the cast, as the reference's bf16 path rounds its operands).  The
    rounding of the inputs shows in s1 as well, so both outputs are held to
    the reference's calibrated bf16 bounds (test_metal_parity.mm:35-38) and
    the north star's 2e-2 relative L2."""
    z = np.load(path)
    L, S, H, P, N, G = (int(v) for v in z["shape"])
    prob = oracle.harness_problem(L, S, H, P, N, G, int(z["seed"]), bool(z["long_memory"]))
    ids = z["ids"] if z["ids"].size else None
    for rt in (None, "128"):
        run_tokens(rt)
        y, s1, d = run(ctx, prob, multipass=True, io="f32", compute="bf16", ids=ids)
        assert "tcgen05" in ctx.backend_desc(d)
        for name, got, want in (("y", y, z["y"]), ("s1", s1, z["s1"])):
            c = compare(got, want, BF16_REL, BF16_ABS)
            record(f"golden bf16 {path.stem} {name} runs={rt}", ratio=c["ratio"], rl2=c["rel_l2"])
            assert c["ok"] and c["rel_l2"] <= BF16_RL2, (path.stem, name, rt, c)


@pytest.mark.parametrize("compute", ["bf16", "f32"])
def test_carry_over_many_runs(ctx, oracle, run_tokens, compute):
    """A run boundary every 128 tokens of 8192: 63 runs carried by the carry
    kernel, folded in segments of eight that combine through shared memory
    (the span-entry state of every 128-token span), on both tensor-core
    families."""
    shape = (8192, 1, 2, 64, 128, 1)
    prob = oracle.harness_problem(*shape, 31337, True)
    prob["s0"] = np.random.default_rng(8).normal(0, 0.2, prob["s0"].shape).astype(np.float32)
    io = "bf16" if compute == "bf16" else "f32"
    w = widen(prob, io)
    y_ref, s_ref = _oracle(oracle, w, shape)
    run_tokens("128")
    y, s1, d = run(ctx, prob, multipass=True, io=io, compute=compute)
    assert ctx.plan_info(d).state_runs == 63
    if compute == "bf16":
        check_bf16("bf16 63 carried runs", y, s1, y_ref, s_ref)
    else:
        from gpu_harness import X3_ABS, X3_REL, X3_RL2
        for got, want in ((y, y_ref), (s1, s_ref)):
            c = compare(got, want, X3_REL, X3_ABS)
            assert c["ok"] and c["rel_l2"] <= X3_RL2, c
