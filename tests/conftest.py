import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes on CPU for the oracle)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def tiny_file():
    from enargeia_b200.format import read_enargeia

    return read_enargeia(GOLDEN / "tiny_q8.enargeia")


def cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not cuda_ok():
        pytest.fail("GPU test run without a CUDA device")
    from enargeia_b200 import build, _lib

    build.build()
    _lib.load()
    import torch

    return torch.device("cuda:0")
