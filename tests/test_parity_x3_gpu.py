"""GPU parity of the fp32-class tensor-core family (F32-stored x, B, C;
compute F32 with backend AUTO or SGMMA): every fp32 operand as a bf16 hi + lo
pair, each product as hi.hi + hi.lo + lo.hi with fp32 accumulators and fp32
carried state.  Against the fp64 oracle on the same inputs, through the C ABI.

Cases mirror the exact-fp32 suite: the reference's 22-shape matrix
(tests/test_metal_parity.mm:77-104) x {planned runs, a run boundary every 128
tokens} x {SHORT, LONG} memory regimes (:121-128), the golden vectors, the
full-size fp32 BASELINE configurations, ids, strided x and y, chunks of
extreme decay, and single pass (which has no scratch for the bf16 pairs and
runs on the exact family).

Bounds: the north star's 1e-4 relative L2 for the fp32 path, and ten times
the reference's calibrated fp32 per-element bound (X3_REL / X3_ABS in
gpu_harness) for y and s1 alike."""
import os
from pathlib import Path

import numpy as np
import pytest

from gpu_harness import F32_ABS, F32_REL, X3_ABS, X3_REL, X3_RL2, record, run
from helpers import compare
from helix_b200 import abi

pytestmark = pytest.mark.gpu

SHAPES = [  # reference tests/test_metal_parity.mm:77-104 (all 22 rows), then extra tiles
    (1, 1, 2, 64, 128, 1), (7, 1, 2, 64, 128, 1), (63, 1, 2, 64, 128, 1),
    (64, 1, 2, 64, 128, 1), (65, 1, 2, 64, 128, 1), (127, 1, 2, 64, 128, 1),
    (128, 1, 2, 64, 128, 1), (129, 1, 2, 64, 128, 1), (96, 1, 4, 64, 128, 1),
    (160, 1, 4, 64, 128, 1), (300, 1, 8, 64, 128, 2), (256, 1, 4, 64, 64, 1),
    (256, 1, 4, 128, 128, 1), (256, 1, 4, 128, 256, 1), (256, 1, 4, 64, 256, 1),
    (300, 1, 4, 128, 256, 1), (256, 1, 8, 128, 256, 2), (256, 1, 4, 192, 128, 1),
    (256, 1, 8, 128, 128, 8), (256, 4, 4, 64, 128, 1),
    (1024, 1, 2, 64, 128, 1), (2048, 1, 8, 64, 128, 2),
    # a partial slab (head_dim 72), d_state 192, and enough heads that the
    # planner gives each output CTA a span of several runs
    (200, 1, 2, 72, 128, 1), (300, 2, 4, 64, 192, 2), (2048, 1, 64, 64, 128, 8),
]


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


def check_x3(tag, y, s1, y_ref, s_ref):
    cy = compare(y, y_ref, X3_REL, X3_ABS)
    cs = compare(s1, s_ref, X3_REL, X3_ABS)
    record(tag, y_ratio=cy["ratio"], y_rl2=cy["rel_l2"], s_ratio=cs["ratio"], s_rl2=cs["rel_l2"])
    assert cy["ok"] and cy["rel_l2"] <= X3_RL2, (tag, "y", cy)
    assert cs["ok"] and cs["rel_l2"] <= X3_RL2, (tag, "s1", cs)


def _oracle(oracle, prob, shape, ids=None, threads=1):
    L, S, H, P, N, G = shape
    d = oracle.desc_init(L, S, H, P, N, G)
    args = [prob[k] for k in ("s0", "x", "dt", "A", "B", "C")]
    if threads > 1:
        return oracle.scan_mt(d, *args, ids=ids, threads=threads)
    return oracle.scan(d, *args, ids=ids)


@pytest.mark.parametrize("backend", [abi.HELIX_BACKEND_SGMMA, abi.HELIX_BACKEND_AUTO], ids=["sgmma", "auto"])
@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
@pytest.mark.parametrize("rt", [None, "128"], ids=["planned", "runs128"])
@pytest.mark.parametrize("shape", SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in SHAPES])
def test_parity_x3(ctx, oracle, run_tokens, shape, rt, long_mem, backend):
    if backend == abi.HELIX_BACKEND_AUTO and (rt or long_mem):
        pytest.skip("AUTO resolves to the same kernels: one regime suffices")
    prob = oracle.harness_problem(*shape, 4242, long_mem)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    run_tokens(rt)
    y, s1, d = run(ctx, prob, multipass=True, backend=backend, compute="f32")
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_SGMMA
    assert "three products" in ctx.backend_desc(d)
    check_x3(f"x3 {rt} {'long' if long_mem else 'short'} {shape}", y, s1, y_ref, s_ref)


def test_single_pass_takes_exact_family(ctx, oracle):
    """Single pass has no scratch for the bf16 pairs: the exact fp32 family
    runs, at the reference's own fp32 bound."""
    shape = (300, 1, 4, 64, 128, 1)
    prob = oracle.harness_problem(*shape, 4242, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    y, s1, d = run(ctx, prob, multipass=False, backend=abi.HELIX_BACKEND_SGMMA)
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_REF
    for got, want in ((y, y_ref), (s1, s_ref)):
        c = compare(got, want, F32_REL, F32_ABS)
        assert c["ok"], c


GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_x3(ctx, oracle, run_tokens, path):
    """Against outputs of the reference's own fp64 oracle (committed)."""
    z = np.load(path)
    L, S, H, P, N, G = (int(v) for v in z["shape"])
    prob = oracle.harness_problem(L, S, H, P, N, G, int(z["seed"]), bool(z["long_memory"]))
    ids = z["ids"] if z["ids"].size else None
    for rt in (None, "128"):
        run_tokens(rt)
        y, s1, _ = run(ctx, prob, multipass=True, backend=abi.HELIX_BACKEND_SGMMA, ids=ids)
        check_x3(f"golden x3 {path.stem} runs={rt}", y, s1, z["y"], z["s1"])


@pytest.mark.parametrize("cfg", ["c1", "c2", "c4"])
def test_baseline_configs_x3(ctx, oracle, cfg):
    """Full-size fp32 BASELINE configurations on the BASELINE distributions,
    with a nonzero initial state, on the default path for compute F32."""
    from helix_b200.synth import Shape, make_inputs, to_numpy_f32
    sh = Shape.of(cfg)
    t = make_inputs(sh, seed=1234, s0_std=0.1)
    prob = {k: to_numpy_f32(t[k]) for k in ("s0", "x", "dt", "A", "B", "C")}
    y_ref, s_ref = _oracle(oracle, prob, (sh.L, sh.S, sh.H, sh.P, sh.N, sh.G), threads=os.cpu_count() or 1)
    y, s1, d = run(ctx, prob, multipass=True, compute="f32")
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_SGMMA
    check_x3(f"x3 baseline {cfg}", y, s1, y_ref, s_ref)


def test_ids_and_batched_x3(ctx, oracle, run_tokens):
    shape = (300, 3, 4, 64, 128, 2)
    prob = oracle.harness_problem(*shape, 777, True)
    ids = np.array([2, 0, 1], np.int32)
    y_ref, s_ref = _oracle(oracle, prob, shape, ids=ids)
    run_tokens("128")
    y, s1, _ = run(ctx, prob, multipass=True, compute="f32", ids=ids)
    check_x3("x3 ids", y, s1, y_ref, s_ref)


def _y_padded_head(shape, dev):
    import torch
    S, L, H, P = shape
    return torch.full((S, L, H, P + 1), float("nan"), dtype=torch.float32, device=dev)[..., :P]


def _y_channel_stride(shape, dev):
    import torch
    S, L, H, P = shape
    return torch.full((S, L, H, 2 * P), float("nan"), dtype=torch.float32, device=dev)[..., ::2]


@pytest.mark.parametrize("y_view", [_y_padded_head, _y_channel_stride], ids=["padded_head", "channel_stride"])
def test_strided_y_x3(ctx, oracle, y_view):
    shape = (300, 2, 4, 64, 128, 2)
    prob = oracle.harness_problem(*shape, 99, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    y, s1, _ = run(ctx, prob, multipass=True, compute="f32", y_view=y_view)
    check_x3(f"x3 strided y {y_view.__name__}", y, s1, y_ref, s_ref)


def test_strided_x_x3(ctx, oracle):
    """x read through a view (head rows 2P + 3 floats apart, channels two
    floats apart): the cast kernel's strided path into the bf16 pairs."""
    import torch
    import helix_b200
    shape = (300, 2, 4, 64, 128, 2)
    prob = oracle.harness_problem(*shape, 7, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    L, S, H, P, N, G = shape
    dev = torch.device("cuda:0")
    big = torch.full((S, L, H, 2 * P + 3), float("nan"), device=dev)
    x = big[..., : 2 * P : 2]
    x.copy_(torch.from_numpy(prob["x"]).to(dev))
    t = {k: torch.from_numpy(np.ascontiguousarray(prob[k])).to(dev) for k in ("s0", "dt", "A", "B", "C")}
    y = torch.full((S, L, H, P), float("nan"), device=dev)
    s1 = torch.full_like(t["s0"], float("nan"))
    d = helix_b200.desc_from_tensors(x, t["dt"], t["B"], t["s0"], y, multipass=True, compute="f32")
    assert ctx.supported(d), ctx.last_error()
    assert "three products" in ctx.backend_desc(d)
    scratch = torch.empty(ctx.scratch_size(d), dtype=torch.uint8, device=dev)
    assert ctx.encode(d, t["s0"], x, t["dt"], t["A"], t["B"], t["C"], y, s1, scratch=scratch) == abi.HELIX_OK
    torch.cuda.synchronize()
    check_x3("x3 strided x", y.cpu().numpy(), s1.cpu().numpy(), y_ref, s_ref)


@pytest.mark.parametrize("where", [0, 1, 3], ids=["first_span", "inner_span", "last_span"])
def test_extreme_decay_chunk_x3(ctx, oracle, run_tokens, where):
    """One chunk of head 0 decays by hundreds of nats (softplus(6) ~ 6 per
    token): the mask's in-group split is off there and every factor is a
    decay, so the output stays finite and exact wherever the chunk falls."""
    shape = (2048, 1, 4, 64, 128, 2)
    prob = oracle.harness_problem(*shape, 4242, True)
    t0 = 512 * where + 128
    prob["dt"][:, t0:t0 + 128, 0] = 6.0
    y_ref, s_ref = _oracle(oracle, prob, shape)
    run_tokens("512")
    y, s1, _ = run(ctx, prob, multipass=True, compute="f32")
    assert np.isfinite(y).all() and np.isfinite(s1).all()
    check_x3(f"x3 extreme decay span {where}", y, s1, y_ref, s_ref)


def test_no_device_fault_recorded_x3(ctx):
    import ctypes as C
    code = C.c_uint32(123)
    assert ctx.lib.helix_device_fault(ctx.handle, C.byref(code)) == abi.HELIX_OK
    assert code.value == 0
