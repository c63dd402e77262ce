"""Generates the committed golden vectors from the REFERENCE's own fp64 oracle.

Inputs come from the reference test harness's generator (xorshift64, restated
in oracle/helix_oracle.c: oracle_harness_fill) with the reference's own seeds;
outputs y and s1 come from helix::ref::scan compiled from the reference sources
(oracle/_ref/libhelix_ref.so, built by oracle/Makefile).  The snapshot case
stores the state at chunk boundaries from helix::ref::scan_with_snapshots.

Run from the repo root in the container that has the reference mounted:
    python tests/golden/make_golden.py
Writes tests/golden/*.npz: shape, seed, regime, ids, a SHA-256 of the
generated inputs (pins the restated generator), and the reference outputs
y, s1 (float32) and, for the snapshot case, the boundary states (float64);
tests/golden/diag/*.npz the same for diagonal A.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.oracle import Oracle, Reference, build, diag_desc  # noqa: E402

OUT = Path(__file__).resolve().parent

# (name, L, S, H, P, N, G, seed, long_memory, ids)
# Shapes follow the reference's edge cases (tests/test_algebra.cpp:28-44,
# tests/test_metal_parity.mm:77-104) at sizes that keep each fixture small.
CASES = [
    ("L1_single_token",  1, 1, 2, 64, 128, 1, 12345, False, None),
    ("L7_partial",       7, 1, 2, 64, 128, 1, 12345, False, None),
    ("L63_chunk_m1",    63, 1, 2, 64, 128, 1, 12345, False, None),
    ("L64_exact",       64, 1, 2, 64, 128, 1, 4242, True, None),
    ("L65_chunk_p1",    65, 1, 2, 64, 128, 1, 4242, True, None),
    ("L129_ragged",    129, 1, 2, 64, 128, 1, 4242, True, None),
    ("L300_g2",        300, 1, 4, 64, 128, 2, 4242, True, None),
    ("dstate64",       256, 1, 2, 64, 64, 1, 12345, False, None),
    ("hdim128",        200, 1, 2, 128, 128, 1, 4242, True, None),
    ("hdim192",        160, 1, 1, 192, 128, 1, 4242, True, None),
    ("dstate256",      130, 1, 2, 64, 256, 1, 4242, True, None),
    ("nseq3_ids",      100, 3, 2, 64, 128, 2, 777, True, [2, 0, 1]),
    ("long_carry",     640, 1, 2, 64, 128, 2, 20260905, True, None),
]
SNAP_CASE = ("snapshots", 384, 1, 2, 64, 128, 1, 20260905, True, None)
# Diagonal A (one rate per (head, state); Oracle.harness_problem_diag) into
# tests/golden/diag/: Mamba-2-like heads, Mamba-1-like head_dim-1 heads with
# d_state 16, tiles that straddle heads, d_state 256, ids.
DIAG_CASES = [
    ("diag_L129_p64",      129, 1, 2, 64, 128, 1, 12345, True, None),
    ("diag_mamba1",        200, 2, 96, 1, 16, 1, 4242, True, None),
    ("diag_p32_g2",        100, 1, 4, 32, 64, 2, 777, False, None),
    ("diag_p72_n256",       70, 1, 2, 72, 256, 1, 4242, True, None),
    ("diag_nseq3_ids",      90, 3, 2, 64, 128, 2, 777, True, [2, 0, 1]),
]


def inputs_digest(prob) -> str:
    h = hashlib.sha256()
    for k in ("s0", "x", "dt", "A", "B", "C"):
        h.update(np.ascontiguousarray(prob[k], np.float32).tobytes())
    return h.hexdigest()


def main():
    build()
    o, r = Oracle(), Reference()
    for name, L, S, H, P, N, G, seed, long_mem, ids in CASES + [SNAP_CASE]:
        prob = o.harness_problem(L, S, H, P, N, G, seed, long_mem)
        d = r.desc_init(L, S, H, P, N, G)
        ids_a = None if ids is None else np.asarray(ids, np.int32)
        args = [prob[k] for k in ("s0", "x", "dt", "A", "B", "C")]
        extra = {}
        if name == "snapshots":
            y, s1, snap = r.scan_with_snapshots(d, *args, chunk=64, ids=ids_a)
            extra["snap"] = snap
            extra["chunk"] = np.int32(64)
        else:
            y, s1 = r.scan(d, *args, ids=ids_a)
        np.savez_compressed(
            OUT / f"{name}.npz", shape=np.array([L, S, H, P, N, G], np.int32), seed=np.uint64(seed),
            long_memory=np.int32(long_mem), ids=(ids_a if ids_a is not None else np.zeros(0, np.int32)),
            inputs_sha256=np.array(inputs_digest(prob)), y=y, s1=s1, **extra)
        print(f"{name:18s} L={L} S={S} H={H} P={P} N={N} G={G}  |y|max={np.abs(y).max():.3e}")
    (OUT / "diag").mkdir(exist_ok=True)
    for name, L, S, H, P, N, G, seed, long_mem, ids in DIAG_CASES:
        prob = o.harness_problem_diag(L, S, H, P, N, G, seed, long_mem)
        d = diag_desc(r.desc_init(L, S, H, P, N, G))
        ids_a = None if ids is None else np.asarray(ids, np.int32)
        y, s1 = r.scan(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")], ids=ids_a)
        np.savez_compressed(
            OUT / "diag" / f"{name}.npz", shape=np.array([L, S, H, P, N, G], np.int32), seed=np.uint64(seed),
            long_memory=np.int32(long_mem), ids=(ids_a if ids_a is not None else np.zeros(0, np.int32)),
            inputs_sha256=np.array(inputs_digest(prob)), y=y, s1=s1)
        print(f"{name:18s} L={L} S={S} H={H} P={P} N={N} G={G}  diagonal A  |y|max={np.abs(y).max():.3e}")


if __name__ == "__main__":
    main()
