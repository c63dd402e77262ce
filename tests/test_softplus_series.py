"""The decay kernels evaluate softplus(v) for v <= 20 as
max(v, 0) + 2 atanh(s), s = e^-|v| / (2 + e^-|v|), with the atanh series cut
after the s^15 term (helix_b200/csrc/kernels/common.cuh, softplus_le20).
This checks the truncated series itself against log1p(exp(v)) in float64,
and a float32 evaluation of the same steps against the float32 library form
the oracle uses (reference src/reference/scan_ref.cpp:13-24)."""
import numpy as np


def _series(v, dtype):
    v = v.astype(dtype)
    u = np.exp(-np.abs(v)).astype(dtype)
    s = (u / (dtype(2) + u)).astype(dtype)
    s2 = s * s
    t = dtype(1.0 / 15.0)
    for c in (13, 11, 9, 7, 5, 3, 1):
        t = (t * s2 + dtype(1.0 / c)).astype(dtype)
    return (np.maximum(v, dtype(0)) + dtype(2) * s * t).astype(dtype)


def test_truncation_error_below_2e9():
    v = np.linspace(-40.0, 20.0, 400001)
    ref = np.log1p(np.exp(v))
    got = _series(v, np.float64)
    assert np.max(np.abs(got - ref) / ref) < 2e-9


def test_float32_within_a_few_ulp_of_library_form():
    rng = np.random.default_rng(7)
    v = np.concatenate([rng.uniform(-30, 20, 200000), np.linspace(-5, 5, 10001)]).astype(np.float32)
    lib = np.log1p(np.exp(v.astype(np.float32))).astype(np.float32)
    got = _series(v, np.float32)
    rel = np.abs(got.astype(np.float64) - lib) / lib
    assert np.max(rel) < 8 * np.finfo(np.float32).eps
