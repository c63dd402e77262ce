"""GPU: numerical drift of the carried state across many chunk boundaries.

Mirrors reference tests/test_drift.mm: L=8192 (128 chunks of 64), H=8, P=64,
N=128; the public API is re-run truncated at every 8th boundary and s1 is
compared with the fp64 oracle's boundary snapshot at the fp32 bound; the late
quarter's worst error must stay within 10x of the early quarter's (:190-200).
Both memory regimes, single pass and multipass, the exact fp32 family at the
fp32 bound and the fp32-class tensor-core family (multipass) at its own
bound."""
import numpy as np
import pytest

from gpu_harness import F32_ABS, F32_REL, X3_ABS, X3_REL, record, run
from helix_b200 import abi

pytestmark = pytest.mark.gpu

L, CHUNK, H, P, N = 8192, 64, 8, 64, 128
MODES = [("1pass/short", False, False), ("multipass/short", True, False),
         ("1pass/long", False, True), ("multipass/long", True, True)]
# (backend, per-element bound): exact CUDA-core family; tensor-core family
FAMILIES = {"exact": (abi.HELIX_BACKEND_REF, F32_REL, F32_ABS), "x3": (abi.HELIX_BACKEND_SGMMA, X3_REL, X3_ABS)}


@pytest.mark.parametrize("family", list(FAMILIES))
@pytest.mark.parametrize("mode", MODES, ids=[m[0] for m in MODES])
def test_drift_f32(ctx, oracle, mode, family):
    name, multipass, long_mem = mode
    if family == "x3" and not multipass:
        pytest.skip("single pass runs on the exact family")
    backend, rel, abs_ = FAMILIES[family]
    prob = oracle.harness_problem(L, 1, H, P, N, 1, 20260905, long_mem)
    d = oracle.desc_init(L, 1, H, P, N, 1)
    _, _, snap = oracle.scan_with_snapshots(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")],
                                             chunk=CHUNK)
    n_chunks = L // CHUNK
    drift = []
    for c in range(7, n_chunks, 8):
        Lc = (c + 1) * CHUNK

        def trunc(dd, Lc=Lc):
            dd.n_tok = Lc
        _, s1, _ = run(ctx, prob, multipass=multipass, backend=backend, desc_hook=trunc)
        want = snap[c]
        err = np.abs(s1.ravel().astype(np.float64) - want)
        ratio = (err / (abs_ + rel * np.abs(want))).max()
        assert np.isfinite(s1).all()
        assert ratio <= 1.0, (name, c, ratio)
        drift.append(err.max())
    q = len(drift) // 4
    early, late = max(drift[:q]), max(drift[-q:])
    growth = late / early if early > 0 else 1.0
    record(f"drift {family} {name}", early=early, late=late, growth=growth)
    assert growth < 10.0, (name, drift)
