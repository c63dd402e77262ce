"""GPU parity of the exact-fp32 CUDA-core kernels (backend REF) against the
fp64 oracle, through the C ABI.  (The fp32-class tensor-core family, backend
SGMMA / AUTO, has its own suite: test_parity_x3_gpu.py.)

Mirrors reference tests/test_metal_parity.mm: its 22-shape matrix
(:77-104) x {single pass, multipass, multipass with many runs} x {SHORT, LONG}
memory regimes (:121-128), the reference's calibrated fp32 per-element bound
(:35-38) with s1 always held to it (:214-218), plus the north star's 1e-4
relative-L2 bar.  "Many runs" (HELIX_RUN_TOKENS=128) plays the role of the
reference's tiny-scratch mode: it puts a run boundary every 128 tokens, so the
run-to-run state carry is exercised on every shape longer than one run.
"""
import os
from pathlib import Path

import numpy as np
import pytest

from gpu_harness import F32_ABS, F32_REL, F32_RL2, record, run
from helpers import compare
from helix_b200 import abi

pytestmark = pytest.mark.gpu

SHAPES = [  # (L, S, H, P, N, G) -- reference tests/test_metal_parity.mm:77-104
    (1, 1, 2, 64, 128, 1), (7, 1, 2, 64, 128, 1), (63, 1, 2, 64, 128, 1),
    (64, 1, 2, 64, 128, 1), (65, 1, 2, 64, 128, 1), (127, 1, 2, 64, 128, 1),
    (128, 1, 2, 64, 128, 1), (129, 1, 2, 64, 128, 1), (96, 1, 4, 64, 128, 1),
    (160, 1, 4, 64, 128, 1), (300, 1, 8, 64, 128, 2), (256, 1, 4, 64, 64, 1),
    (256, 1, 4, 128, 128, 1), (256, 1, 4, 128, 256, 1), (256, 1, 4, 64, 256, 1),
    (300, 1, 4, 128, 256, 1), (256, 1, 8, 128, 256, 2), (256, 1, 4, 192, 128, 1),
    (256, 1, 8, 128, 128, 8), (256, 4, 4, 64, 128, 1), (1024, 1, 2, 64, 128, 1),
    (2048, 1, 8, 64, 128, 2),
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


def _check(tag, y, s1, y_ref, s_ref):
    cy = compare(y, y_ref, F32_REL, F32_ABS)
    cs = compare(s1, s_ref, F32_REL, F32_ABS)
    record(tag, y_ratio=cy["ratio"], y_rl2=cy["rel_l2"], s_ratio=cs["ratio"], s_rl2=cs["rel_l2"])
    assert cy["ok"] and cy["rel_l2"] <= F32_RL2, (tag, "y", cy)
    assert cs["ok"] and cs["rel_l2"] <= F32_RL2, (tag, "s1", cs)


@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
@pytest.mark.parametrize("mode", MODES, ids=[m[0] for m in MODES])
@pytest.mark.parametrize("shape", SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in SHAPES])
def test_parity_f32(ctx, oracle, run_tokens, shape, mode, long_mem):
    L, S, H, P, N, G = shape
    name, multipass, rt = mode
    prob = oracle.harness_problem(L, S, H, P, N, G, 4242, long_mem)
    d = oracle.desc_init(L, S, H, P, N, G)
    y_ref, s_ref = oracle.scan(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")])
    run_tokens(rt)
    y, s1, dd = run(ctx, prob, multipass=multipass, backend=abi.HELIX_BACKEND_REF)
    assert ctx.select_backend(dd) == abi.HELIX_BACKEND_REF
    _check(f"f32 {name} {'long' if long_mem else 'short'} {shape}", y, s1, y_ref, s_ref)


GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_f32(ctx, oracle, run_tokens, path):
    """Against outputs of the reference's own fp64 oracle (committed)."""
    z = np.load(path)
    L, S, H, P, N, G = (int(v) for v in z["shape"])
    prob = oracle.harness_problem(L, S, H, P, N, G, int(z["seed"]), bool(z["long_memory"]))
    ids = z["ids"] if z["ids"].size else None
    for rt in (None, "128"):
        run_tokens(rt)
        y, s1, _ = run(ctx, prob, multipass=True, backend=abi.HELIX_BACKEND_REF, ids=ids)
        _check(f"golden {path.stem} runs={rt}", y, s1, z["y"], z["s1"])


@pytest.mark.parametrize("cfg", ["c1", "c2", "c4"])
def test_baseline_configs_f32(ctx, oracle, cfg):
    """Full-size fp32 BASELINE configurations on the BASELINE distributions,
    with a nonzero initial state to exercise the carry-in."""
    from helix_b200.synth import Shape, make_inputs, to_numpy_f32
    sh = Shape.of(cfg)
    t = make_inputs(sh, seed=1234, s0_std=0.1)
    prob = {k: to_numpy_f32(t[k]) for k in ("s0", "x", "dt", "A", "B", "C")}
    d = oracle.desc_init(sh.L, sh.S, sh.H, sh.P, sh.N, sh.G)
    y_ref, s_ref = oracle.scan_mt(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")],
                                  threads=os.cpu_count() or 1)
    y, s1, _ = run(ctx, prob, multipass=True, compute="f32", backend=abi.HELIX_BACKEND_REF)
    _check(f"baseline {cfg}", y, s1, y_ref, s_ref)
