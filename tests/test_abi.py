"""CPU: the C-ABI library loads, exports every symbol include/helix/helix.h
declares, and its host-only behaviour matches the reference's."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from helix_b200 import abi

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    out = []
    for hdr in sorted((ROOT / "include").rglob("*.h")):
        txt = re.sub(r"/\*.*?\*/", "", hdr.read_text(), flags=re.S)
        out += re.findall(r"\b(helix_\w+)\s*\(", txt)
    inline = {"helix_tensor_is_null"}
    return sorted(set(out) - inline)


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    syms = declared_symbols()
    assert set(abi.EXPORTS) <= set(syms)
    for s in syms:
        assert hasattr(lib, s), s


def test_struct_layout_matches_reference(reference):
    assert C.sizeof(abi.ScanDesc) == reference.desc_size()


@pytest.mark.parametrize("shape", [(512, 1, 64, 64, 128, 8), (1000, 4, 32, 192, 128, 1), (1, 3, 2, 8, 16, 2)])
def test_desc_init_matches_reference(reference, shape):
    ours = abi.desc_init(*shape)
    theirs = reference.desc_init(*shape)
    assert bytes(ours) == bytes(theirs)


def test_null_handling_without_device():
    lib = abi.load()
    d = abi.desc_init(64, 1, 2, 64, 128, 1)
    assert lib.helix_scan_supported(None, C.byref(d)) is False
    assert lib.helix_ctx_backend_desc(None, C.byref(d)) == b"unavailable (null context)"
    assert lib.helix_ctx_select_backend(None, C.byref(d)) == abi.HELIX_BACKEND_REF
    assert lib.helix_ctx_last_error(None)
    # single pass needs no scratch, whatever the context
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == 0
    st = lib.helix_scan_encode(None, None, C.byref(d), *([abi.NULL_TENSOR] * 10))
    assert st == abi.HELIX_ERR_INVALID_ARG
    assert lib.helix_ctx_create(None, None, None) == abi.HELIX_ERR_INVALID_ARG


def test_ctx_create_reports_no_device_here():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    lib = abi.load()
    h = C.c_void_p()
    assert lib.helix_ctx_create(C.byref(h), None, None) == abi.HELIX_ERR_NO_DEVICE
    assert not h.value


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError):
        abi.load(tmp_path / "libhelix.so")


def test_tensor_core_scratch_plan_c3():
    """BASELINE config 3 (bf16 operands, multipass) on a 148-SM part: spans of
    16 chunks (4 output spans, 128 pair tiles), 2 runs per span chosen by the
    state kernel's cost model, so 6 run states per head are kept, plus one
    log-decay per run state, one path record per output tile and one decay
    span per run (8 per head), each region 256-byte aligned."""
    lib = abi.load()
    d = abi.desc_init(8192, 1, 64, 64, 128, 8)
    d.io_dtype = 2  # HELIX_BF16
    d.compute_dtype = 2
    d.multipass = True

    def al(n):
        return (n + 255) // 256 * 256

    agg = 64 * 6 * 64 * 128 * 4
    lam = al(64 * 6 * 4)
    flags = al(8 * 4 * 4 * 4)
    spans = al(64 * 8 * 4)
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == agg + lam + flags + spans


def test_fp32_tensor_core_scratch_plan_c2():
    """BASELINE config 2 (F32-stored x, B, C; compute F32: the three-product
    tensor-core family) on a 148-SM part: one 64-channel slab per output CTA,
    two output spans of 8 chunks (128 CTAs), the first span cut into 4 runs of
    256 tokens for the state kernel; scratch = 4 run states and log-decays per
    head, then bf16 hi and lo copies of B and C.  x is read in place (dense
    fp32), so there is no x copy; a view of x TMA cannot describe (channels two
    floats apart) adds a dense fp32 copy."""
    lib = abi.load()

    def desc():
        d = abi.desc_init(2048, 1, 64, 64, 128, 8)
        d.io_dtype = 0  # HELIX_F32
        d.compute_dtype = 0
        d.multipass = True
        return d

    def al(n):
        return (n + 255) // 256 * 256

    agg = al(64 * 4 * 64 * 128 * 4)
    lam = al(64 * 4 * 4)
    bc = al(2048 * 8 * 128 * 2)
    d = desc()
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == agg + lam + 4 * bc
    d = desc()
    d.s_x[2] = 2  # channels two floats apart
    d.s_x[1] = 2 * 64
    d.s_x[0] = 64 * 2 * 64
    d.seq_x = 2048 * 64 * 2 * 64
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == agg + lam + al(2048 * 64 * 64 * 4) + 4 * bc


def test_diagonal_a_scratch_plan():
    """Diagonal A (one rate per (head, state)) on a 148-SM part: one output
    CTA per 64 (head, channel) rows of a group, runs cut so the output kernel
    has about four CTAs per SM; scratch = one run state and one dt sum per run
    before the last, no copies.  Config 3's shape: 64 tiles -> 10 runs of 896
    tokens; a Mamba-1 layer (2048 heads of head_dim 1, d_state 16, one group):
    32 tiles -> 16 runs of 512 tokens; single pass needs none."""
    lib = abi.load()

    def al(n):
        return (n + 255) // 256 * 256

    def desc(L, S, H, P, N, G, multipass=True):
        d = abi.desc_init(L, S, H, P, N, G)
        d.a_form = abi.HELIX_A_DIAG_PER_CHANNEL
        d.s_a = N
        d.multipass = multipass
        return d

    d = desc(8192, 1, 64, 64, 128, 8)
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == al(64 * 9 * 64 * 128 * 4) + al(64 * 9 * 4)
    d = desc(8192, 1, 2048, 1, 16, 1)
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == al(2048 * 15 * 1 * 16 * 4) + al(2048 * 15 * 4)
    d = desc(8192, 1, 64, 64, 128, 8, multipass=False)
    assert lib.helix_scan_scratch_size(None, C.byref(d)) == 0
