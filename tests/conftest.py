import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_vectors.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built native library")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA; run with -m 'not gpu'")
    return torch.device("cuda:0")


os.environ.setdefault("OMP_NUM_THREADS", str(min(8, os.cpu_count() or 1)))
