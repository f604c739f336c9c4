"""Host-side bridges (no GPU): numpy <-> torch Arrays, as in the reference's
tests/test_bridges.py (to_numpy passthrough, to_torch from numpy)."""

import numpy as np
import torch

from scree_b200 import Array
from scree_b200.bridges import to_numpy, to_torch


def test_to_torch_from_numpy_zero_copy():
    vals = np.arange(12, dtype=np.float32).reshape(6, 2)
    arr = Array(values=vals, offsets=np.array([0, 2, 6], dtype=np.int64))
    t = to_torch(arr)
    assert isinstance(t.values, torch.Tensor) and t.offsets.dtype == torch.int32
    vals[0, 0] = 42.0  # shares memory with the numpy source
    assert float(t.values[0, 0]) == 42.0


def test_to_numpy_passthrough():
    arr = Array(values=np.zeros((3, 1)), offsets=np.array([0, 3]))
    assert to_numpy(arr) is arr
    t = Array(values=torch.ones((4, 2)), offsets=torch.tensor([0, 1, 4]))
    n = to_numpy(t)
    assert isinstance(n.values, np.ndarray) and n.offsets.tolist() == [0, 1, 4]
