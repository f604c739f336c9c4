import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def load_golden(name):
    with np.load(GOLDEN / f"golden_{name}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def decode16(bits, dtype):
    """uint16 bit patterns -> float64 values."""
    dtype = str(dtype)
    if dtype == "float16":
        return bits.view(np.float16).astype(np.float64)
    if dtype == "bfloat16":
        return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return bits.astype(np.float64)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from scree_b200 import _lib

    _lib.load()
    return torch.device("cuda:0")
