"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

* ``Oracle``     -- our C restatement (oracle/liboracle.so, helix_oracle.c)
* ``Reference``  -- the reference's own fp64 oracle compiled from its sources
                    (oracle/_ref/libhelix_ref.so), when it has been built

Both take numpy float32 arrays in the helix.h layouts and a helix_b200.abi
ScanDesc.  Nothing here is used by the shipped library.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

from helix_b200.abi import ScanDesc

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libhelix_ref.so"

_F = C.POINTER(C.c_float)
_I = C.POINTER(C.c_int32)
_D = C.POINTER(C.c_double)


# Where the reference checkout is mounted in the build container; the GPU box
# has no reference and uses the prebuilt oracle/_ref.  HELIX_REF_ROOT overrides.
REF_MOUNT = "/root/reference"


def build() -> None:
    """Runs oracle/Makefile (builds _ref too when the reference sources exist)."""
    ref = os.environ.get("HELIX_REF_ROOT", REF_MOUNT)
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF_ROOT={ref}"], check=True)


def _f(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def _ids(ids):
    if ids is None:
        return None
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    return ids.ctypes.data_as(_I)


class _Base:
    prefix = ""

    def __init__(self, path: Path):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (python -c 'import oracle.oracle as o; o.build()')")
        self.lib = C.CDLL(str(path))
        sig = [C.POINTER(ScanDesc), _F, _F, _F, _F, _F, _F, _I, _F, _F]
        for name in ("scan", "scan_chunked"):
            fn = getattr(self.lib, self.prefix + name)
            fn.argtypes = sig
        self._snap = getattr(self.lib, self.prefix + self.snap_name)
        self._snap.argtypes = sig + [C.c_int32, _D]

    def _run(self, fn, d, s0, x, dt, A, B, Cm, ids, y=None, s1=None):
        y = np.zeros((d.n_seq, d.n_tok, d.n_head, d.head_dim), np.float32) if y is None else y
        s1 = np.zeros((d.n_seq, d.n_head, d.head_dim, d.d_state), np.float32) if s1 is None else s1
        keep = [np.ascontiguousarray(a, dtype=np.float32) for a in (s0, x, dt, A, B, Cm)]
        ia = None if ids is None else np.ascontiguousarray(ids, dtype=np.int32)
        fn(C.byref(d), *[_f(a) for a in keep], _ids(ia), _f(y), _f(s1))
        return y, s1

    def scan(self, d, s0, x, dt, A, B, Cm, ids=None):
        return self._run(getattr(self.lib, self.prefix + "scan"), d, s0, x, dt, A, B, Cm, ids)

    def scan_chunked(self, d, s0, x, dt, A, B, Cm, ids=None):
        return self._run(getattr(self.lib, self.prefix + "scan_chunked"), d, s0, x, dt, A, B, Cm, ids)

    def scan_with_snapshots(self, d, s0, x, dt, A, B, Cm, chunk, ids=None):
        n_chunks = (d.n_tok + chunk - 1) // chunk
        snap = np.zeros((n_chunks, d.n_seq * d.seq_s), np.float64)
        y = np.zeros((d.n_seq, d.n_tok, d.n_head, d.head_dim), np.float32)
        s1 = np.zeros((d.n_seq, d.n_head, d.head_dim, d.d_state), np.float32)
        keep = [np.ascontiguousarray(a, dtype=np.float32) for a in (s0, x, dt, A, B, Cm)]
        ia = None if ids is None else np.ascontiguousarray(ids, dtype=np.int32)
        self._snap(C.byref(d), *[_f(a) for a in keep], _ids(ia), _f(y), _f(s1), chunk,
                   snap.ctypes.data_as(_D))
        return y, s1, snap


class Oracle(_Base):
    """Our C restatement (oracle/helix_oracle.c)."""
    prefix = "oracle_"
    snap_name = "scan_snapshots"

    def __init__(self, path: Path = ORACLE_SO):
        super().__init__(path)
        L = self.lib
        L.oracle_scan_mt.argtypes = [C.POINTER(ScanDesc), _F, _F, _F, _F, _F, _F, _I, _F, _F, C.c_int32]
        L.oracle_scan_chunked.restype = C.c_int
        L.oracle_desc_init.argtypes = [C.POINTER(ScanDesc)] + [C.c_int32] * 6
        L.oracle_harness_fill.argtypes = [C.c_int32] * 6 + [C.c_uint64, C.c_int32] + [_F] * 6
        L.oracle_carry_chain.argtypes = [C.c_int32, C.c_int64, _D, _D, _D, _D]

    def scan_mt(self, d, s0, x, dt, A, B, Cm, ids=None, threads: int = 1):
        y = np.zeros((d.n_seq, d.n_tok, d.n_head, d.head_dim), np.float32)
        s1 = np.zeros((d.n_seq, d.n_head, d.head_dim, d.d_state), np.float32)
        keep = [np.ascontiguousarray(a, dtype=np.float32) for a in (s0, x, dt, A, B, Cm)]
        ia = None if ids is None else np.ascontiguousarray(ids, dtype=np.int32)
        self.lib.oracle_scan_mt(C.byref(d), *[_f(a) for a in keep], _ids(ia), _f(y), _f(s1), threads)
        return y, s1

    def desc_init(self, L, S, H, P, N, G) -> ScanDesc:
        d = ScanDesc()
        self.lib.oracle_desc_init(C.byref(d), L, S, H, P, N, G)
        return d

    def harness_problem(self, L, S, H, P, N, G, seed, long_memory=False):
        """Inputs exactly as the reference test harness makes them
        (reference tests/harness.hpp:151-186)."""
        s0 = np.zeros((S, H, P, N), np.float32)
        x = np.zeros((S, L, H, P), np.float32)
        dt = np.zeros((S, L, H), np.float32)
        A = np.zeros((H,), np.float32)
        B = np.zeros((S, L, G, N), np.float32)
        Cm = np.zeros((S, L, G, N), np.float32)
        self.lib.oracle_harness_fill(L, S, H, P, N, G, seed, int(long_memory),
                                     *[_f(a) for a in (s0, x, dt, A, B, Cm)])
        return dict(s0=s0, x=x, dt=dt, A=A, B=B, C=Cm)

    def harness_problem_diag(self, L, S, H, P, N, G, seed, long_memory=False):
        """The harness problem with diagonal A (one rate per (head, state),
        helix.h HELIX_A_DIAG_PER_CHANNEL, read as A[h * d_state + n]): each
        head's harness rate times a factor drawn log-uniform in [1/4, 4]
        (numpy PCG64 seeded with `seed`), so both memory regimes keep their
        decay scale.  The reference's harness has no diagonal-A generator."""
        prob = self.harness_problem(L, S, H, P, N, G, seed, long_memory)
        f = np.exp(np.random.default_rng(seed).uniform(-np.log(4.0), np.log(4.0), (H, N)))
        prob["A"] = (prob["A"][:, None] * f).astype(np.float32)
        return prob

    def carry_chain(self, s0, agg, lam):
        """carry[k] = state entering slice k (see helix_oracle.c)."""
        K = agg.shape[0]
        s0 = np.ascontiguousarray(s0, np.float64).reshape(-1)
        agg = np.ascontiguousarray(agg, np.float64).reshape(K, -1)
        lam = np.ascontiguousarray(lam, np.float64).reshape(K)
        out = np.zeros_like(agg)
        self.lib.oracle_carry_chain(K, agg.shape[1], s0.ctypes.data_as(_D), agg.ctypes.data_as(_D),
                                    lam.ctypes.data_as(_D), out.ctypes.data_as(_D))
        return out


class Reference(_Base):
    """The reference's own fp64 oracle (helix::ref), compiled from its sources."""
    prefix = "ref_"
    snap_name = "scan_with_snapshots"

    def __init__(self, path: Path = REF_SO):
        super().__init__(path)
        self.lib.ref_desc_init.argtypes = [C.POINTER(ScanDesc)] + [C.c_int32] * 6
        self.lib.ref_desc_size.restype = C.c_int

    def desc_init(self, L, S, H, P, N, G) -> ScanDesc:
        d = ScanDesc()
        self.lib.ref_desc_init(C.byref(d), L, S, H, P, N, G)
        return d

    def desc_size(self) -> int:
        return int(self.lib.ref_desc_size())


def diag_desc(d):
    """Switches a dense descriptor to diagonal A (A dense [n_head][d_state])."""
    d.a_form = 1  # HELIX_A_DIAG_PER_CHANNEL
    d.s_a = d.d_state
    return d


def available_reference() -> bool:
    return REF_SO.exists()
