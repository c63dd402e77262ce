"""The ggml-cuda bridge (integration/ggml/ggml-helix-cuda.cpp), the CUDA
counterpart of the reference's ggml-metal hook
(reference integration/ggml/ggml-helix.cpp:157-361).

CPU: it compiles (-Wall -Wextra, against the field-level stand-in in
integration/ggml/compat/) and exports the hook.
GPU: the hook is called the way ggml-cuda's SSM_SCAN would call it, with
ggml-shaped tensors (fastest dimension first, byte strides, dst holding y and
then the final state) built over torch buffers; it must serve the op (on the
fp32-class tensor-core family, the bridge's default) and match the fp64
oracle within that family's bounds, and decline -- returning false with dst untouched --
what the reference bridge declines: K > 1 snapshots, non-F32 tensors, a
per-channel A, fewer than the minimum tokens (32, measured: profiles/length_gate.md)."""
import ctypes as C

import numpy as np
import pytest

from gpu_harness import X3_ABS, X3_REL, X3_RL2
from helpers import compare

GGML_F32, GGML_I32, GGML_OTHER = 0, 1, 2


class GgmlTensor(C.Structure):
    """integration/ggml/compat/ggml.h"""
    _fields_ = [("type", C.c_int), ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4), ("op_params", C.c_int32 * 16),
                ("src", C.c_void_p * 8), ("data", C.c_void_p)]


@pytest.fixture(scope="module")
def bridge():
    from integration.ggml.build import build
    lib = C.CDLL(str(build()))
    lib.ggml_cuda_op_ssm_scan_helix.argtypes = [C.c_void_p, C.c_int, C.POINTER(GgmlTensor)]
    lib.ggml_cuda_op_ssm_scan_helix.restype = C.c_bool
    return lib


def test_bridge_compiles_and_exports_the_hook(bridge):
    assert hasattr(bridge, "ggml_cuda_op_ssm_scan_helix")


def _view(t, shape_fast_first, dtype_size=4, typ=GGML_F32):
    """A ggml tensor over torch tensor t: ne fastest first, nb in bytes."""
    g = GgmlTensor()
    g.type = typ
    ne = list(shape_fast_first) + [1] * (4 - len(shape_fast_first))
    g.ne[:] = ne
    nb = [dtype_size]
    for k in range(1, 4):
        nb.append(nb[-1] * ne[k - 1])
    g.nb[:] = nb
    g.data = t.data_ptr()
    return g


def _op(t, L, S, H, P, N, G, K=1, a_diag=False, x_type=GGML_F32):
    """ggml's SSM_SCAN node over torch tensors t (dense helix.h layouts)."""
    srcs = [_view(t["s0"], [N, P, H, S]), _view(t["x"], [P, H, L, S], typ=x_type), _view(t["dt"], [H, L, S]),
            _view(t["A"], [N if a_diag else 1, H]), _view(t["B"], [N, G, L, S]), _view(t["C"], [N, G, L, S]),
            _view(t["ids"], [S], typ=GGML_I32)]
    dst = _view(t["dst"], [P * H * L * S + N * P * H * S])
    dst.op_params[0] = K
    for k, s in enumerate(srcs):
        dst.src[k] = C.addressof(s)
    dst._keep = srcs
    return dst


def _tensors(oracle, L, S, H, P, N, G, a_diag=False):
    import torch
    dev = torch.device("cuda:0")
    make = oracle.harness_problem_diag if a_diag else oracle.harness_problem
    prob = make(L, S, H, P, N, G, 4242, True)  # diagonal A: [H][N]
    prob["s0"] = np.random.default_rng(1).normal(0, 0.1, prob["s0"].shape).astype(np.float32)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in prob.items()}
    t["ids"] = torch.arange(S, dtype=torch.int32, device=dev).flip(0).contiguous()  # reversed rows
    t["dst"] = torch.full((S * L * H * P + S * H * P * N,), float("nan"), device=dev)
    return prob, t


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(300, 2, 8, 64, 128, 2), (1000, 1, 4, 128, 128, 1), (512, 1, 4, 64, 256, 2)],
                         ids=["L300", "L1000P128", "N256"])
def test_bridge_serves_ssm_scan(bridge, oracle, shape):
    import torch
    L, S, H, P, N, G = shape
    prob, t = _tensors(oracle, *shape)
    dst = _op(t, *shape)
    stream = torch.cuda.current_stream().cuda_stream
    assert bridge.ggml_cuda_op_ssm_scan_helix(C.c_void_p(stream), 0, C.byref(dst))
    torch.cuda.synchronize()
    out = t["dst"].cpu().numpy()
    y = out[: S * L * H * P].reshape(S, L, H, P)
    s1 = out[S * L * H * P:].reshape(S, H, P, N)
    d = oracle.desc_init(*shape)
    ids = t["ids"].cpu().numpy()
    y_ref, s_ref = oracle.scan(d, *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")], ids=ids)
    for got, want in ((y, y_ref), (s1, s_ref)):
        c = compare(got, want, X3_REL, X3_ABS)
        assert c["ok"] and c["rel_l2"] <= X3_RL2, c


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(300, 2, 8, 64, 128, 2), (200, 2, 96, 1, 16, 1)], ids=["mamba2_like", "mamba1_like"])
def test_bridge_serves_diagonal_a(bridge, oracle, shape):
    """A {d_state, n_head} (one rate per state): the reference's hook
    declines it; this one runs the diagonal-A recurrence kernels."""
    import torch
    from oracle.oracle import diag_desc
    L, S, H, P, N, G = shape
    prob, t = _tensors(oracle, *shape, a_diag=True)
    dst = _op(t, *shape, a_diag=True)
    stream = torch.cuda.current_stream().cuda_stream
    assert bridge.ggml_cuda_op_ssm_scan_helix(C.c_void_p(stream), 0, C.byref(dst))
    torch.cuda.synchronize()
    out = t["dst"].cpu().numpy()
    y = out[: S * L * H * P].reshape(S, L, H, P)
    s1 = out[S * L * H * P:].reshape(S, H, P, N)
    ids = t["ids"].cpu().numpy()
    y_ref, s_ref = oracle.scan(diag_desc(oracle.desc_init(*shape)),
                               *[prob[k] for k in ("s0", "x", "dt", "A", "B", "C")], ids=ids)
    for got, want in ((y, y_ref), (s1, s_ref)):
        c = compare(got, want, X3_REL, X3_ABS)
        assert c["ok"] and c["rel_l2"] <= X3_RL2, c


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["K2", "f16_x", "short"])
def test_bridge_declines_what_the_reference_declines(bridge, oracle, case):
    import torch
    shape = (31 if case == "short" else 300, 1, 4, 64, 128, 1)
    _, t = _tensors(oracle, *shape)
    dst = _op(t, *shape, K=2 if case == "K2" else 1, x_type=GGML_OTHER if case == "f16_x" else GGML_F32)
    stream = torch.cuda.current_stream().cuda_stream
    assert not bridge.ggml_cuda_op_ssm_scan_helix(C.c_void_p(stream), 0, C.byref(dst))
    torch.cuda.synchronize()
    assert bool(torch.isnan(t["dst"]).all()), "nothing may be enqueued when the hook declines"
