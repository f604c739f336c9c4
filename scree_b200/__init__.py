"""scree_b200 — B200-native (sm_100a) varlen hot path with scree's API.

Drop-in for scree's packed-sequence primitive (scree/__init__.py:3-22) and the
GPU kernels behind scree.kernels: Array, pack, unpack, to_padded, from_padded,
from_cu_seqlens, and scree_b200.kernels (Array-level) /
scree_b200.kernels.triton (tensor-level names).  All data-moving ops run
hand-written CUDA kernels from libscree_b200.so; there is no CPU path.
"""

from ._core import Array, from_cu_seqlens, from_padded, pack, to_padded, unpack
from . import kernels

__version__ = "0.1.0"

__all__ = [
    "Array",
    "pack",
    "unpack",
    "to_padded",
    "from_padded",
    "from_cu_seqlens",
    "kernels",
    "__version__",
]
