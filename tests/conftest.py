import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")
    config.addinivalue_line("markers", "slow: long CPU test")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import ORACLE_SO, Oracle, build
    if not ORACLE_SO.exists():
        build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, available_reference, build
    if not available_reference():
        build()
    if not available_reference():
        pytest.skip("reference oracle (oracle/_ref) not built here")
    return Reference()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ctx(cuda):
    import helix_b200
    return helix_b200.Context(0)
