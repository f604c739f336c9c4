"""Drop-in module path for code written against scree.kernels.triton.

scree/kernels/triton/__init__.py:10-31 exports the GPU entry points and a
TRITON_AVAILABLE flag.  This package keeps that import path and those names so
``from scree_b200.kernels.triton import varlen_attention_triton`` works
unchanged, but nothing here uses Triton: every name is the sm_100a CUDA
implementation from scree_b200.kernels.native.  TRITON_AVAILABLE reports
whether that native library is present (the reference's meaning: "the GPU
kernels can be called").
"""

from .._native_flag import NATIVE_AVAILABLE as TRITON_AVAILABLE
from ..native import (
    varlen_attention_triton,
    varlen_attention_triton_autograd,
    varlen_attention_triton_backward,
    varlen_layernorm_triton,
    varlen_rmsnorm_triton,
)

__all__ = [
    "varlen_attention_triton",
    "varlen_attention_triton_autograd",
    "varlen_layernorm_triton",
    "varlen_rmsnorm_triton",
    "TRITON_AVAILABLE",
]
