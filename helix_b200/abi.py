"""ctypes mirror of include/helix/helix.h.

Field order, types and enum values follow the C header exactly; the header in
turn keeps the reference ABI (reference include/helix/helix.h:42-218).
``load()`` opens the in-tree ``libhelix.so`` and raises when it is missing: the
package has no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhelix.so"

# helix_status
HELIX_OK = 0
HELIX_ERR_UNSUPPORTED_SHAPE = 1
HELIX_ERR_NO_DEVICE = 2
HELIX_ERR_SCRATCH_TOO_SMALL = 3
HELIX_ERR_INVALID_ARG = 4
HELIX_ERR_PIPELINE = 5
STATUS_NAMES = {0: "OK", 1: "UNSUPPORTED_SHAPE", 2: "NO_DEVICE", 3: "SCRATCH_TOO_SMALL",
                4: "INVALID_ARG", 5: "PIPELINE"}

# helix_dtype
HELIX_F32, HELIX_F16, HELIX_BF16 = 0, 1, 2
# helix_a_form
HELIX_A_SCALAR_PER_HEAD, HELIX_A_DIAG_PER_CHANNEL = 0, 1
# helix_backend
HELIX_BACKEND_AUTO, HELIX_BACKEND_SGMMA, HELIX_BACKEND_MPP, HELIX_BACKEND_REF = 0, 1, 2, 3

I32, I64 = C.c_int32, C.c_int64


class ScanDesc(C.Structure):
    """helix_scan_desc."""
    _fields_ = [
        ("n_tok", I32), ("n_seq", I32), ("n_head", I32), ("head_dim", I32),
        ("d_state", I32), ("n_group", I32),
        ("s_x", I64 * 3), ("s_b", I64 * 3), ("s_c", I64 * 3), ("s_dt", I64 * 2),
        ("s_s", I64 * 3), ("s_y", I64 * 3), ("s_a", I64),
        ("seq_x", I64), ("seq_b", I64), ("seq_c", I64), ("seq_dt", I64),
        ("seq_s", I64), ("seq_y", I64),
        ("chunk", I32), ("a_form", C.c_int), ("io_dtype", C.c_int),
        ("compute_dtype", C.c_int), ("backend", C.c_int), ("multipass", C.c_bool),
        ("dt_min", C.c_float), ("dt_max", C.c_float),
    ]

    def copy(self) -> "ScanDesc":
        d = ScanDesc()
        C.memmove(C.byref(d), C.byref(self), C.sizeof(ScanDesc))
        return d


class Tensor(C.Structure):
    """helix_tensor: device pointer + byte offset."""
    _fields_ = [("buf", C.c_void_p), ("offset", C.c_uint64)]


NULL_TENSOR = Tensor(None, 0)

# Every entry point include/helix/*.h declares.
EXPORTS = (
    "helix_scan_desc_init", "helix_ctx_create", "helix_ctx_free", "helix_ctx_last_error",
    "helix_ctx_select_backend", "helix_ctx_backend_desc", "helix_scan_supported",
    "helix_scan_scratch_size", "helix_scan_encode", "helix_scan_encode_into",
    # include/helix/helix_ext.h
    "helix_device_fault", "helix_scan_encode_static",
    "helix_scan_shard_state_scratch_size", "helix_scan_shard_state", "helix_scan_carry_combine",
    "helix_scan_plan_info", "helix_scan_encode_shard",
)


class PlanInfo(C.Structure):
    """helix_plan_info (include/helix/helix_ext.h)."""
    _fields_ = [("family", I32), ("chunk", I32), ("run_tokens", I32), ("n_runs", I32),
                ("runs_per_span", I32), ("n_spans", I32), ("state_runs", I32), ("reserved", I32),
                ("scratch_bytes", C.c_uint64)]

_lib = None


def load(path: Path | str | None = None) -> C.CDLL:
    """Opens libhelix.so and declares prototypes.  Raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `python -m helix_b200.build`")
    lib = C.CDLL(str(p))
    P = C.POINTER
    lib.helix_scan_desc_init.argtypes = [P(ScanDesc), I32, I32, I32, I32, I32, I32]
    lib.helix_scan_desc_init.restype = None
    lib.helix_ctx_create.argtypes = [P(C.c_void_p), C.c_void_p, C.c_char_p]
    lib.helix_ctx_create.restype = C.c_int
    lib.helix_ctx_free.argtypes = [C.c_void_p]
    lib.helix_ctx_free.restype = None
    lib.helix_ctx_last_error.argtypes = [C.c_void_p]
    lib.helix_ctx_last_error.restype = C.c_char_p
    lib.helix_ctx_select_backend.argtypes = [C.c_void_p, P(ScanDesc)]
    lib.helix_ctx_select_backend.restype = C.c_int
    lib.helix_ctx_backend_desc.argtypes = [C.c_void_p, P(ScanDesc)]
    lib.helix_ctx_backend_desc.restype = C.c_char_p
    lib.helix_scan_supported.argtypes = [C.c_void_p, P(ScanDesc)]
    lib.helix_scan_supported.restype = C.c_bool
    lib.helix_scan_scratch_size.argtypes = [C.c_void_p, P(ScanDesc)]
    lib.helix_scan_scratch_size.restype = C.c_size_t
    enc = [C.c_void_p, C.c_void_p, P(ScanDesc)] + [Tensor] * 10
    lib.helix_scan_encode.argtypes = enc
    lib.helix_scan_encode.restype = C.c_int
    lib.helix_scan_encode_into.argtypes = enc
    lib.helix_scan_encode_into.restype = C.c_int
    lib.helix_device_fault.argtypes = [C.c_void_p, P(C.c_uint32)]
    lib.helix_device_fault.restype = C.c_int
    lib.helix_scan_encode_static.argtypes = [C.c_void_p, C.c_void_p, P(ScanDesc)] + [Tensor] * 9
    lib.helix_scan_encode_static.restype = C.c_int
    lib.helix_scan_shard_state_scratch_size.argtypes = [C.c_void_p, P(ScanDesc)]
    lib.helix_scan_shard_state_scratch_size.restype = C.c_size_t
    lib.helix_scan_shard_state.argtypes = [C.c_void_p, C.c_void_p, P(ScanDesc)] + [Tensor] * 8
    lib.helix_scan_shard_state.restype = C.c_int
    lib.helix_scan_carry_combine.argtypes = [C.c_void_p, C.c_void_p, P(ScanDesc)] + [Tensor] * 4 + [
        C.c_uint32, Tensor]
    lib.helix_scan_carry_combine.restype = C.c_int
    lib.helix_scan_encode_shard.argtypes = [C.c_void_p, C.c_void_p, P(ScanDesc)] + [Tensor] * 9
    lib.helix_scan_encode_shard.restype = C.c_int
    lib.helix_scan_plan_info.argtypes = [C.c_void_p, P(ScanDesc), P(PlanInfo)]
    lib.helix_scan_plan_info.restype = C.c_int
    if path is None:
        _lib = lib
    return lib


def desc_init(L: int, S: int, H: int, P: int, N: int, G: int) -> ScanDesc:
    d = ScanDesc()
    load().helix_scan_desc_init(C.byref(d), L, S, H, P, N, G)
    return d
