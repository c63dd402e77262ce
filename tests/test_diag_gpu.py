"""GPU parity of the diagonal-A family (a_form HELIX_A_DIAG_PER_CHANNEL: one
decay rate per (head, state), Mamba-1's selective scan), against the fp64
oracle through the C ABI.

The reference declines diagonal A on the GPU (src/runtime/caps.mm:121-123);
its fp64 oracle runs it (src/reference/scan_ref.cpp:27-29), and the
restatement here matches that oracle bit for bit (tests/test_oracle.py,
golden vectors in tests/golden/diag).  The kernels run the recurrence in fp32,
so the bound is the fp32 one used for the fp32-class tensor-core family: the
north star's 1e-4 relative L2 for the fp32 path and ten times the
reference's calibrated fp32 per-element bound (X3_REL / X3_ABS), for y and
s1 alike.  bf16-stored x, B, C are checked against the oracle fed the same
bf16-rounded values.

Cases: Mamba-2-like heads (a 64-row tile inside one head, decays staged once
per token), head_dim-1 heads of Mamba-1 (a tile spans 64 heads), tiles that
straddle heads, d_state from 8 to 256, each in single pass, planned runs and
a run boundary every 128 tokens, both memory regimes, both storage dtypes;
the golden vectors; ids; strided x and y; a chunk of extreme decay; every
backend and precision request; the token-shard entry points, which need a
scalar decay and decline."""
import os
from pathlib import Path

import numpy as np
import pytest

from gpu_harness import X3_ABS, X3_REL, X3_RL2, record, run, widen
from helpers import compare
from helix_b200 import abi
from oracle.oracle import diag_desc

pytestmark = pytest.mark.gpu

SHAPES = [  # (L, S, H, P, N, G)
    (1, 1, 2, 64, 128, 1), (63, 1, 2, 64, 128, 1), (129, 1, 2, 64, 128, 1),
    (300, 1, 8, 64, 128, 2), (256, 1, 4, 128, 256, 1), (256, 4, 4, 64, 64, 1),
    (1024, 1, 2, 64, 128, 1), (300, 2, 96, 1, 16, 1), (200, 1, 4, 32, 64, 2),
    (150, 1, 2, 72, 128, 1), (100, 1, 3, 48, 8, 1), (130, 2, 8, 16, 20, 4),
]
MODES = [("1pass", False, None), ("multipass", True, None), ("runs128", True, "128")]


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


def _diag_hook(d):
    diag_desc(d)


def _oracle(oracle, prob, shape, ids=None):
    args = [prob[k] for k in ("s0", "x", "dt", "A", "B", "C")]
    return oracle.scan(diag_desc(oracle.desc_init(*shape)), *args, ids=ids)


def _check(tag, y, s1, y_ref, s_ref):
    cy = compare(y, y_ref, X3_REL, X3_ABS)
    cs = compare(s1, s_ref, X3_REL, X3_ABS)
    record(tag, y_ratio=cy["ratio"], y_rl2=cy["rel_l2"], s_ratio=cs["ratio"], s_rl2=cs["rel_l2"])
    assert cy["ok"] and cy["rel_l2"] <= X3_RL2, (tag, "y", cy)
    assert cs["ok"] and cs["rel_l2"] <= X3_RL2, (tag, "s1", cs)


@pytest.mark.parametrize("io", ["f32", "bf16"])
@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
@pytest.mark.parametrize("mode", MODES, ids=[m[0] for m in MODES])
@pytest.mark.parametrize("shape", SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in SHAPES])
def test_parity_diag(ctx, oracle, run_tokens, shape, mode, long_mem, io):
    tag, multipass, rt = mode
    prob = oracle.harness_problem_diag(*shape, 4242, long_mem)
    prob["s0"] = np.random.default_rng(5).normal(0, 0.1, prob["s0"].shape).astype(np.float32)
    y_ref, s_ref = _oracle(oracle, widen(prob, io), shape)
    run_tokens(rt)
    y, s1, d = run(ctx, prob, multipass=multipass, io=io, desc_hook=_diag_hook)
    assert ctx.select_backend(d) == abi.HELIX_BACKEND_REF
    assert "diagonal A" in ctx.backend_desc(d)
    _check(f"diag {io} {tag} {'long' if long_mem else 'short'} {shape}", y, s1, y_ref, s_ref)


GOLDEN = sorted((Path(__file__).parent / "golden" / "diag").glob("*.npz"))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_diag(ctx, oracle, run_tokens, path):
    """Against outputs of the reference's own fp64 oracle (committed)."""
    z = np.load(path)
    L, S, H, P, N, G = (int(v) for v in z["shape"])
    prob = oracle.harness_problem_diag(L, S, H, P, N, G, int(z["seed"]), bool(z["long_memory"]))
    ids = z["ids"] if z["ids"].size else None
    for multipass, rt in ((False, None), (True, None), (True, "128")):
        run_tokens(rt)
        y, s1, _ = run(ctx, prob, multipass=multipass, ids=ids, desc_hook=_diag_hook)
        _check(f"golden diag {path.stem} mp={multipass} runs={rt}", y, s1, z["y"], z["s1"])


@pytest.mark.parametrize("backend,compute", [(abi.HELIX_BACKEND_AUTO, "bf16"), (abi.HELIX_BACKEND_SGMMA, "f32"),
                                             (abi.HELIX_BACKEND_MPP, "f32"), (abi.HELIX_BACKEND_REF, "f32")],
                         ids=["auto_bf16", "sgmma", "mpp", "ref"])
def test_every_request_takes_the_recurrence(ctx, oracle, backend, compute):
    """Whatever backend and precision are asked for, diagonal A runs the fp32
    recurrence (no reassociated, reduced-precision form exists for it)."""
    shape = (300, 1, 4, 64, 128, 2)
    prob = oracle.harness_problem_diag(*shape, 777, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    y, s1, d = run(ctx, prob, multipass=True, backend=backend, compute=compute, desc_hook=_diag_hook)
    assert "diagonal A" in ctx.backend_desc(d)
    _check(f"diag backend {backend} {compute}", y, s1, y_ref, s_ref)


def test_mamba1_model_shape(ctx, oracle):
    """A Mamba-1 layer's scan: d_inner 1536 head_dim-1 heads, d_state 16,
    one group, two sequences of 1024 tokens."""
    shape = (1024, 2, 1536, 1, 16, 1)
    prob = oracle.harness_problem_diag(*shape, 20260905, False)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    y, s1, d = run(ctx, prob, multipass=True, desc_hook=_diag_hook)
    _check("diag mamba1 1536x16", y, s1, y_ref, s_ref)


def test_ids_and_batched_diag(ctx, oracle, run_tokens):
    shape = (300, 3, 4, 64, 128, 2)
    prob = oracle.harness_problem_diag(*shape, 777, True)
    prob["s0"] = np.random.default_rng(3).normal(0, 0.1, prob["s0"].shape).astype(np.float32)
    ids = np.array([2, 0, 1], np.int32)
    y_ref, s_ref = _oracle(oracle, prob, shape, ids=ids)
    run_tokens("128")
    y, s1, _ = run(ctx, prob, multipass=True, ids=ids, desc_hook=_diag_hook)
    _check("diag ids", y, s1, y_ref, s_ref)


def test_strided_x_and_y_diag(ctx, oracle):
    """x read through a view (head rows 2P + 3 floats apart, channels two
    floats apart) and y written through a channel-strided view."""
    import torch
    import helix_b200
    shape = (200, 2, 4, 64, 64, 2)
    prob = oracle.harness_problem_diag(*shape, 7, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    L, S, H, P, N, G = shape
    dev = torch.device("cuda:0")
    big = torch.full((S, L, H, 2 * P + 3), float("nan"), device=dev)
    x = big[..., : 2 * P : 2]
    x.copy_(torch.from_numpy(prob["x"]).to(dev))
    t = {k: torch.from_numpy(np.ascontiguousarray(prob[k])).to(dev) for k in ("s0", "dt", "A", "B", "C")}
    y = torch.full((S, L, H, 2 * P), float("nan"), device=dev)[..., ::2]
    s1 = torch.full_like(t["s0"], float("nan"))
    d = helix_b200.desc_from_tensors(x, t["dt"], t["B"], t["s0"], y, multipass=True, A=t["A"])
    assert d.a_form == abi.HELIX_A_DIAG_PER_CHANNEL and d.s_a == N
    assert ctx.supported(d), ctx.last_error()
    scratch = torch.empty(max(ctx.scratch_size(d), 256), dtype=torch.uint8, device=dev)
    assert ctx.encode(d, t["s0"], x, t["dt"], t["A"], t["B"], t["C"], y, s1, scratch=scratch) == abi.HELIX_OK
    torch.cuda.synchronize()
    _check("diag strided x, y", y.cpu().numpy(), s1.cpu().numpy(), y_ref, s_ref)


def test_padded_a_rows(ctx, oracle):
    """A read through a view whose head rows are d_state + 3 floats apart
    (s_a = d_state + 3): the kernels index A[h * s_a + n]."""
    import torch
    import helix_b200
    shape = (300, 1, 4, 32, 64, 2)  # head_dim 32: tiles span two heads (per-lane rates)
    L, S, H, P, N, G = shape
    prob = oracle.harness_problem_diag(*shape, 5, True)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    dev = torch.device("cuda:0")
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
    big = torch.full((H, N + 3), float("nan"), device=dev)
    A = big[:, :N]
    A.copy_(t["A"])
    y, s1 = helix_b200.scan(t["x"], t["dt"], A, t["B"], t["C"], t["s0"], ctx=ctx)
    torch.cuda.synchronize()
    _check("diag padded A rows", y.cpu().numpy(), s1.cpu().numpy(), y_ref, s_ref)
    for uni_shape in ((300, 1, 2, 64, 64, 1),):  # head_dim 64: one head per tile (staged decays)
        prob = oracle.harness_problem_diag(*uni_shape, 6, True)
        y_ref, s_ref = _oracle(oracle, prob, uni_shape)
        t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
        big = torch.full((uni_shape[2], uni_shape[4] + 3), float("nan"), device=dev)
        A = big[:, :uni_shape[4]]
        A.copy_(t["A"])
        y, s1 = helix_b200.scan(t["x"], t["dt"], A, t["B"], t["C"], t["s0"], ctx=ctx)
        torch.cuda.synchronize()
        _check("diag padded A rows, one head per tile", y.cpu().numpy(), s1.cpu().numpy(), y_ref, s_ref)


def test_high_level_scan_reads_the_a_form(oracle):
    """helix_b200.scan takes A of shape (n_head, d_state) as diagonal A."""
    import torch
    import helix_b200
    shape = (256, 1, 4, 64, 32, 1)
    prob = oracle.harness_problem_diag(*shape, 99, False)
    y_ref, s_ref = _oracle(oracle, prob, shape)
    dev = torch.device("cuda:0")
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
    y, s1 = helix_b200.scan(t["x"], t["dt"], t["A"], t["B"], t["C"], t["s0"])
    torch.cuda.synchronize()
    _check("diag helix_b200.scan", y.cpu().numpy(), s1.cpu().numpy(), y_ref, s_ref)


@pytest.mark.parametrize("where", [0, 2], ids=["first_run", "inner_run"])
def test_extreme_decay_diag(ctx, oracle, run_tokens, where):
    """A chunk of head 0 decays by hundreds of nats (softplus(6) ~ 6 per
    token, rates up to 64): states vanish there and come back finite."""
    shape = (1024, 1, 4, 64, 128, 2)
    prob = oracle.harness_problem_diag(*shape, 4242, True)
    t0 = 256 * where + 64
    prob["dt"][:, t0:t0 + 128, 0] = 6.0
    y_ref, s_ref = _oracle(oracle, prob, shape)
    run_tokens("256")
    y, s1, _ = run(ctx, prob, multipass=True, desc_hook=_diag_hook)
    assert np.isfinite(y).all() and np.isfinite(s1).all()
    _check(f"diag extreme decay {where}", y, s1, y_ref, s_ref)


def test_token_shards_decline_diagonal_a(ctx, oracle):
    """The L-split entry points exchange one log-decay per (seq, head): only
    scalar A has one, so they decline diagonal A and enqueue nothing."""
    import torch
    import helix_b200
    shape = (256, 1, 4, 64, 64, 1)
    prob = oracle.harness_problem_diag(*shape, 1, False)
    dev = torch.device("cuda:0")
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
    with pytest.raises(helix_b200.HelixError) as e:
        helix_b200.shard_state(t["x"], t["dt"], t["A"], t["B"], t["C"])
    assert "scalar A" in str(e.value)


def test_no_device_fault_recorded_diag(ctx):
    import ctypes as C
    code = C.c_uint32(123)
    assert ctx.lib.helix_device_fault(ctx.handle, C.byref(code)) == abi.HELIX_OK
    assert code.value == 0
