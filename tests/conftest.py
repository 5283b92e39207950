import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def golden_cpu():
    return np.load(GOLDEN / "reference_cpu.npz")


@pytest.fixture(scope="session")
def golden_gpu():
    path = GOLDEN / "reference_gpu.npz"
    if not path.exists():
        pytest.skip("reference_gpu.npz not generated yet (tests/golden/make_golden.py gpu)")
    return np.load(path)


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for gpu-marked tests.  On a machine with a GPU the
    extension must be built: a missing extension is an error, not a skip."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from code_for_iclr27_b200 import operators

    operators()
    return torch.device("cuda:0")
