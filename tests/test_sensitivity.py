"""CPU: the parity bounds catch the kernel mistakes they exist to catch.

The reference's README claims mutation testing against seeded kernel bugs,
with no harness in the repository; its harness notes that a 1.002x error in
the carried state went unnoticed under the SHORT memory regime, which is why
the LONG regime exists (reference tests/harness.hpp:130-140).  Mistakes are
planted here in the oracle, on the CPU, as a kernel would make them, and the
bounds the GPU parity suites use must reject the result:
* the state carried across a run boundary scaled by 1.002 (LONG regime);
* the decay of one chunk applied once too often (a dropped boundary term);
* dt read one token late;
* the bf16 family's bound against a carry that skipped one run.
Each mutated output is compared with the unmutated oracle at the bound that
suite uses; the test passes when the comparison fails."""
import numpy as np
import pytest

from gpu_harness import BF16_ABS, BF16_REL, F32_ABS, F32_REL, X3_ABS, X3_REL
from helpers import compare

SHAPE = (512, 1, 2, 64, 128, 1)  # L, S, H, P, N, G
BOUNDS = {"exact fp32": (F32_REL, F32_ABS), "fp32-class tensor cores": (X3_REL, X3_ABS)}


def _args(prob):
    return [prob[k] for k in ("s0", "x", "dt", "A", "B", "C")]


def _slice(prob, t0, t1, s0):
    out = dict(prob)
    for k in ("x", "dt", "B", "C"):
        out[k] = np.ascontiguousarray(prob[k][:, t0:t1])
    out["s0"] = np.ascontiguousarray(s0, np.float32)
    return out


def _split_scan(oracle, prob, cut, mutate):
    """Scans [0, cut) and [cut, L) separately, passing the state through
    mutate() at the boundary, as a kernel's run carry does."""
    L, S, H, P, N, G = SHAPE
    _, mid = oracle.scan(oracle.desc_init(cut, S, H, P, N, G), *_args(_slice(prob, 0, cut, prob["s0"])))
    y2, s2 = oracle.scan(oracle.desc_init(L - cut, S, H, P, N, G),
                         *_args(_slice(prob, cut, L, mutate(mid, prob, cut))))
    return y2, s2


@pytest.mark.parametrize("bound", list(BOUNDS), ids=["f32", "x3"])
def test_carry_scaled_by_1_002_is_caught_in_the_long_regime(oracle, bound):
    prob = oracle.harness_problem(*SHAPE, 4242, True)
    y_ref, s_ref = oracle.scan(oracle.desc_init(*SHAPE), *_args(prob))
    cut = 256
    # unmutated split: identical to the whole scan at round-off
    y_ok, _ = _split_scan(oracle, prob, cut, lambda s, p, c: s)
    assert compare(y_ok, y_ref[:, cut:], *BOUNDS[bound])["ok"]
    y_bad, s_bad = _split_scan(oracle, prob, cut, lambda s, p, c: s * 1.002)
    cy = compare(y_bad, y_ref[:, cut:], *BOUNDS[bound])
    cs = compare(s_bad, s_ref, *BOUNDS[bound])
    assert not (cy["ok"] and cs["ok"]), (cy, cs)


def test_one_extra_chunk_decay_is_caught(oracle):
    """The boundary state decayed by one more chunk's factor (a doubled
    exp(Lc_end) at a run boundary)."""
    prob = oracle.harness_problem(*SHAPE, 777, True)
    y_ref, s_ref = oracle.scan(oracle.desc_init(*SHAPE), *_args(prob))
    cut = 256

    def extra_decay(s, p, c):
        dt = np.log1p(np.exp(p["dt"][0, c - 64:c].astype(np.float64)))  # last 64 tokens' softplus
        f = np.exp((dt * p["A"][None, :]).sum(0))  # [H]
        return s * f[None, :, None, None]
    y_bad, s_bad = _split_scan(oracle, prob, cut, extra_decay)
    assert not compare(y_bad, y_ref[:, cut:], F32_REL, F32_ABS)["ok"]
    assert not compare(s_bad, s_ref, F32_REL, F32_ABS)["ok"]


@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
def test_dt_one_token_late_is_caught(oracle, long_mem):
    prob = oracle.harness_problem(*SHAPE, 12345, long_mem)
    y_ref, _ = oracle.scan(oracle.desc_init(*SHAPE), *_args(prob))
    bad = dict(prob)
    bad["dt"] = np.ascontiguousarray(np.concatenate([prob["dt"][:, :1], prob["dt"][:, :-1]], axis=1))
    y_bad, _ = oracle.scan(oracle.desc_init(*SHAPE), *_args(bad))
    for rel, ab in BOUNDS.values():
        assert not compare(y_bad, y_ref, rel, ab)["ok"]


def test_skipped_run_is_caught_even_at_the_bf16_bound(oracle):
    """The bf16 family's y bound is loose (1.5e-2), but a carry that drops a
    whole run's contribution still fails it, and s1 is held to fp32 bounds."""
    prob = oracle.harness_problem(*SHAPE, 4242, True)
    y_ref, s_ref = oracle.scan(oracle.desc_init(*SHAPE), *_args(prob))
    cut = 256
    y_bad, s_bad = _split_scan(oracle, prob, cut, lambda s, p, c: np.zeros_like(s))
    cy = compare(y_bad, y_ref[:, cut:], BF16_REL, BF16_ABS)
    cs = compare(s_bad, s_ref, 2e-5, 2e-6)
    assert not cy["ok"] and not cs["ok"]
