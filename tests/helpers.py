"""Shared test utilities: error metrics and problem construction."""
from __future__ import annotations

import numpy as np


def compare(got, ref, rel_tol, abs_tol):
    """Per-element allclose ratio of reference tests/harness.hpp:63-83:
    worst |a-b| / (abs_tol + rel_tol*|b|); pass iff <= 1 and all finite."""
    a = np.asarray(got, np.float64).ravel()
    b = np.asarray(ref, np.float64).ravel()
    if not (np.isfinite(a).all() and np.isfinite(b).all()):
        return dict(ok=False, finite=False, ratio=np.inf, max_abs=np.inf, rel_l2=np.inf)
    err = np.abs(a - b)
    ratio = err / (abs_tol + rel_tol * np.abs(b)) if a.size else np.zeros(0)
    rl2 = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)) if a.size else 0.0
    worst = float(ratio.max()) if a.size else 0.0
    return dict(ok=worst <= 1.0, finite=True, ratio=worst, max_abs=float(err.max()) if a.size else 0.0,
                rel_l2=rl2, at=int(ratio.argmax()) if a.size else -1)


def rel_l2(got, ref) -> float:
    a = np.asarray(got, np.float64).ravel()
    b = np.asarray(ref, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def dense_desc(oracle, L, S, H, P, N, G, chunk=0):
    d = oracle.desc_init(L, S, H, P, N, G)
    d.chunk = chunk
    return d
