"""CPU: pin the C restatement (oracle/helix_oracle.c) to the reference.

1. Golden vectors (tests/golden/*.npz) hold y, s1 and boundary states that the
   REFERENCE's own fp64 oracle produced; the restated input generator must
   reproduce the recorded inputs (checksum) and the restatement must reproduce
   the outputs.  These run anywhere (no reference checkout needed).
2. Where the reference oracle is built here (oracle/_ref), the restatement is
   compared with it directly on the reference's shape matrix
   (reference tests/test_algebra.cpp:28-44) in both memory regimes.
3. The algebraic facts the reference pins: chunked == sequential at f32
   round-off (rel 1e-6 / abs 1e-9, test_algebra.cpp:49-50) and chunk
   invariance over 16..256 (test_algebra.cpp:80-93).
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from helpers import compare

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))
ALG_REL, ALG_ABS = 1e-6, 1e-9


def _load(path):
    z = np.load(path)
    L, S, H, P, N, G = (int(v) for v in z["shape"])
    return z, (L, S, H, P, N, G)


def _digest(prob):
    h = hashlib.sha256()
    for k in ("s0", "x", "dt", "A", "B", "C"):
        h.update(np.ascontiguousarray(prob[k], np.float32).tobytes())
    return h.hexdigest()


def _args(prob):
    return [prob[k] for k in ("s0", "x", "dt", "A", "B", "C")]


def test_golden_files_present():
    assert len(GOLDEN) >= 10


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden(oracle, path):
    z, (L, S, H, P, N, G) = _load(path)
    prob = oracle.harness_problem(L, S, H, P, N, G, int(z["seed"]), bool(z["long_memory"]))
    assert _digest(prob) == str(z["inputs_sha256"]), "restated input generator drifted"
    ids = z["ids"] if z["ids"].size else None
    d = oracle.desc_init(L, S, H, P, N, G)
    if "snap" in z.files:
        y, s1, snap = oracle.scan_with_snapshots(d, *_args(prob), chunk=int(z["chunk"]), ids=ids)
        np.testing.assert_array_equal(snap, z["snap"])
    else:
        y, s1 = oracle.scan(d, *_args(prob), ids=ids)
    # Same fp64 arithmetic in the same order: the f32 results must match
    # the reference's bit for bit.
    np.testing.assert_array_equal(y, z["y"])
    np.testing.assert_array_equal(s1, z["s1"])


ALG_SHAPES = [  # reference tests/test_algebra.cpp:28-44
    (1, 1, 1, 64, 128, 1, 64), (7, 1, 2, 64, 128, 1, 64), (63, 1, 2, 64, 128, 1, 64),
    (64, 1, 2, 64, 128, 1, 64), (65, 1, 2, 64, 128, 1, 64), (127, 1, 2, 64, 128, 1, 64),
    (128, 1, 2, 64, 128, 1, 64), (129, 1, 2, 64, 128, 1, 64), (256, 1, 4, 64, 64, 1, 64),
    (256, 1, 4, 128, 128, 1, 64), (256, 1, 8, 128, 128, 8, 64), (256, 4, 4, 64, 128, 1, 64),
    (512, 1, 2, 64, 128, 1, 32), (512, 1, 2, 64, 128, 1, 128), (1024, 1, 2, 64, 128, 1, 64),
]


@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
@pytest.mark.parametrize("shape", ALG_SHAPES, ids=[f"L{s[0]}S{s[1]}H{s[2]}P{s[3]}N{s[4]}G{s[5]}c{s[6]}" for s in ALG_SHAPES])
def test_restatement_vs_reference(oracle, reference, shape, long_mem):
    L, S, H, P, N, G, chunk = shape
    prob = oracle.harness_problem(L, S, H, P, N, G, 12345, long_mem)
    d = oracle.desc_init(L, S, H, P, N, G)
    d.chunk = chunk
    rd = reference.desc_init(L, S, H, P, N, G)
    rd.chunk = chunk
    assert bytes(d) == bytes(rd), "desc_init differs from the reference's"
    y_o, s_o = oracle.scan(d, *_args(prob))
    y_r, s_r = reference.scan(rd, *_args(prob))
    np.testing.assert_array_equal(y_o, y_r)
    np.testing.assert_array_equal(s_o, s_r)
    yc_o, sc_o = oracle.scan_chunked(d, *_args(prob))
    yc_r, sc_r = reference.scan_chunked(rd, *_args(prob))
    assert compare(yc_o, yc_r, ALG_REL, ALG_ABS)["ok"]
    assert compare(sc_o, sc_r, ALG_REL, ALG_ABS)["ok"]
    # the algebra itself: chunked == sequential at f32 round-off
    assert compare(yc_o, y_o, ALG_REL, ALG_ABS)["ok"]
    assert compare(sc_o, s_o, ALG_REL, ALG_ABS)["ok"]


def test_chunk_invariance(oracle):
    ref = None
    for chunk in (16, 32, 64, 128, 256):
        prob = oracle.harness_problem(509, 1, 4, 64, 128, 1, 777, False)
        d = oracle.desc_init(509, 1, 4, 64, 128, 1)
        d.chunk = chunk
        y, s = oracle.scan_chunked(d, *_args(prob))
        if ref is None:
            ref = (y, s)
            continue
        assert compare(y, ref[0], ALG_REL, ALG_ABS)["ok"], chunk
        assert compare(s, ref[1], ALG_REL, ALG_ABS)["ok"], chunk


def test_threaded_driver_is_bit_identical(oracle):
    prob = oracle.harness_problem(200, 2, 6, 64, 128, 3, 4242, True)
    d = oracle.desc_init(200, 2, 6, 64, 128, 3)
    y1, s1 = oracle.scan(d, *_args(prob))
    y4, s4 = oracle.scan_mt(d, *_args(prob), threads=4)
    np.testing.assert_array_equal(y1, y4)
    np.testing.assert_array_equal(s1, s4)


def test_carry_chain_is_the_sequential_state(oracle):
    """Cutting a slice into K pieces, scanning each from a zero state and
    chaining (exp(lam), agg) reproduces the uncut final state: the identity the
    library's runs and the multi-GPU L-split rely on."""
    L, H, P, N, K = 384, 2, 64, 64, 3
    prob = oracle.harness_problem(L, 1, H, P, N, 1, 4242, True)
    d = oracle.desc_init(L, 1, H, P, N, 1)
    _, s_full = oracle.scan(d, *_args(prob))
    piece = L // K
    aggs, lams = [], []
    zero = np.zeros_like(prob["s0"])
    for k in range(K):
        sl = slice(k * piece, (k + 1) * piece)
        sub = dict(prob, x=np.ascontiguousarray(prob["x"][:, sl]), dt=np.ascontiguousarray(prob["dt"][:, sl]),
                   B=np.ascontiguousarray(prob["B"][:, sl]), C=np.ascontiguousarray(prob["C"][:, sl]), s0=zero)
        dk = oracle.desc_init(piece, 1, H, P, N, 1)
        _, agg = oracle.scan(dk, *_args(sub))
        aggs.append(agg.astype(np.float64))
        dtk = np.log1p(np.exp(prob["dt"][0, sl].astype(np.float64)))
        lams.append((dtk * prob["A"].astype(np.float64)[None, :]).sum(0))  # [H]
    # per-head chain (lam is per head): run it head by head
    for h in range(H):
        carry = oracle.carry_chain(prob["s0"][0, h].astype(np.float64),
                                   np.stack([a[0, h] for a in aggs]), np.array([l[h] for l in lams]))
        final = np.exp(lams[-1][h]) * carry[-1] + aggs[-1][0, h].ravel()
        assert compare(final, s_full[0, h].ravel(), 1e-5, 1e-7)["ok"]


# ---- diagonal A (HELIX_A_DIAG_PER_CHANNEL) ----------------------------------

GOLDEN_DIAG = sorted((Path(__file__).parent / "golden" / "diag").glob("*.npz"))


def test_golden_diag_files_present():
    assert len(GOLDEN_DIAG) >= 5


@pytest.mark.parametrize("path", GOLDEN_DIAG, ids=[p.stem for p in GOLDEN_DIAG])
def test_golden_diag(oracle, path):
    """Diagonal-A outputs of the reference's own fp64 oracle (its scan reads
    A[h * s_a + n] for this form, src/reference/scan_ref.cpp:27-29)."""
    from oracle.oracle import diag_desc
    z, (L, S, H, P, N, G) = _load(path)
    prob = oracle.harness_problem_diag(L, S, H, P, N, G, int(z["seed"]), bool(z["long_memory"]))
    assert _digest(prob) == str(z["inputs_sha256"]), "restated input generator drifted"
    ids = z["ids"] if z["ids"].size else None
    y, s1 = oracle.scan(diag_desc(oracle.desc_init(L, S, H, P, N, G)), *_args(prob), ids=ids)
    np.testing.assert_array_equal(y, z["y"])
    np.testing.assert_array_equal(s1, z["s1"])


DIAG_SHAPES = [(1, 1, 1, 64, 128, 1), (65, 1, 2, 64, 128, 1), (130, 2, 64, 1, 16, 1),
               (100, 1, 4, 48, 64, 2), (64, 1, 2, 64, 256, 1)]


@pytest.mark.parametrize("long_mem", [False, True], ids=["short", "long"])
@pytest.mark.parametrize("shape", DIAG_SHAPES, ids=["L{}S{}H{}P{}N{}G{}".format(*s) for s in DIAG_SHAPES])
def test_diag_restatement_vs_reference(oracle, reference, shape, long_mem):
    from oracle.oracle import diag_desc
    prob = oracle.harness_problem_diag(*shape, 12345, long_mem)
    y_o, s_o = oracle.scan(diag_desc(oracle.desc_init(*shape)), *_args(prob))
    y_r, s_r = reference.scan(diag_desc(reference.desc_init(*shape)), *_args(prob))
    np.testing.assert_array_equal(y_o, y_r)
    np.testing.assert_array_equal(s_o, s_r)
    # the chunked reassociation has no diagonal form: both decline it
    y_c, _ = oracle.scan_chunked(diag_desc(oracle.desc_init(*shape)), *_args(prob))
    assert not np.any(y_c)


def test_diag_run_carry_identity(oracle):
    """Cutting a slice into K runs, scanning each from a zero state and
    chaining S = exp(A[h][n] D_k) S + agg_k, D_k the run's dt sum, reproduces
    the uncut final state: the identity the diagonal-A kernels' run carry
    relies on (A is constant over a run, so a state's decay over it is one
    exponential of the summed dt)."""
    from oracle.oracle import diag_desc
    L, H, P, N, K = 384, 2, 8, 16, 3
    prob = oracle.harness_problem_diag(L, 1, H, P, N, 1, 4242, True)
    _, s_full = oracle.scan(diag_desc(oracle.desc_init(L, 1, H, P, N, 1)), *_args(prob))
    piece = L // K
    zero = np.zeros_like(prob["s0"])
    state = prob["s0"][0].astype(np.float64)  # [H][P][N]
    A = prob["A"].astype(np.float64)          # [H][N]
    for k in range(K):
        sl = slice(k * piece, (k + 1) * piece)
        sub = dict(prob, x=np.ascontiguousarray(prob["x"][:, sl]), dt=np.ascontiguousarray(prob["dt"][:, sl]),
                   B=np.ascontiguousarray(prob["B"][:, sl]), C=np.ascontiguousarray(prob["C"][:, sl]), s0=zero)
        _, agg = oracle.scan(diag_desc(oracle.desc_init(piece, 1, H, P, N, 1)), *_args(sub))
        D = np.log1p(np.exp(prob["dt"][0, sl].astype(np.float64))).sum(0)  # [H]
        state = np.exp(A * D[:, None])[:, None, :] * state + agg[0].astype(np.float64)
    assert compare(state.astype(np.float32), s_full[0], 1e-5, 1e-7)["ok"]
