"""GPU: the tcgen05 operand layouts (K-major / MN-major, TMA- and
thread-written, 128-byte swizzle) used by the tensor-core kernels, each
checked as one 128x128x128 bf16 GEMM against torch in fp32."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def probe():
    from tests.native.build import build
    lib = C.CDLL(str(build()))
    lib.umma_probe.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    return lib


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_umma_layout(probe, cuda, mode):
    g = torch.Generator(device="cpu").manual_seed(mode)
    P = torch.randn(128, 128, generator=g).to(torch.bfloat16).to(cuda)
    Q = torch.randn(128, 128, generator=g).to(torch.bfloat16).to(cuda)
    n = 128 if mode in (0, 1, 4) else 64
    D = torch.full((128, n), float("nan"), device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = probe.umma_probe(mode, P.data_ptr(), Q.data_ptr(), D.data_ptr(), status.data_ptr())
    assert rc == 0
    assert int(status.item()) == 0, "bounded wait expired"
    Pf, Qf = P.float(), Q.float()
    want = {0: Pf @ Qf.T, 1: Pf @ Qf.T, 2: Pf @ Qf[:, :64], 3: Pf.T @ Qf[:, :64], 4: Pf @ Qf.T}[mode]
    err = (D - want).abs().max().item()
    assert err <= 1e-3 * want.abs().max().item(), (mode, err)
