import os
import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "flashinfer-bench-starter-kit_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity tests want every data-dependent kernel error surfaced as an exception.
os.environ.setdefault("DSA_B200_CHECK", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
