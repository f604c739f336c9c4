"""Array-level varlen kernels (the scree.kernels.reference signatures) on the GPU.

Same call shapes as scree/kernels/reference/__init__.py:7-17 for the hot path:
  varlen_attention(q, k, v, causal=False) -> Array   reference/varlen_attention.py:10
  varlen_rmsnorm(arr, weight=None, eps=1e-6) -> Array reference/varlen_rmsnorm.py:18
  varlen_layernorm(arr, weight=None, bias=None, eps=1e-5) -> Array
                                                      reference/varlen_layernorm.py:14
  varlen_softmax(arr) -> Array                        reference/varlen_softmax.py:13
Every call runs the sm_100a kernels of libscree_b200 and is differentiable
(torch autograd), like the reference's torch branch.  Output Arrays reuse the
input's offsets object (reference/varlen_attention.py:140).
"""

from __future__ import annotations

from .._core import Array, _is_torch
from . import native

__all__ = ["varlen_attention", "varlen_rmsnorm", "varlen_layernorm", "varlen_softmax", "native"]


def _check_cuda(arr: Array, name: str) -> None:
    if not (_is_torch(arr.values) and arr.values.is_cuda):
        raise TypeError(f"scree_b200.kernels.{name} requires CUDA torch tensors")


def varlen_attention(q: Array, k: Array, v: Array, causal: bool = False) -> Array:
    """Varlen self-attention, scale 1/sqrt(head_dim); q, k, v (T, H, D) with
    head_dim 32, 64 or 128.  fp16 / bf16 run on the tcgen05 tensor-core kernels;
    fp32 (the reference's Array-level default, reference/varlen_attention.py:90-114)
    runs on fp32 CUDA-core kernels with fp32-grade results."""
    import torch

    for a in (q, k, v):
        _check_cuda(a, "varlen_attention")
    if not (q.offsets is k.offsets and q.offsets is v.offsets):
        if not (torch.equal(q.offsets, k.offsets) and torch.equal(q.offsets, v.offsets)):
            raise ValueError("q, k, v must have identical offsets")
    if q.values.dtype == torch.float32:
        out = native.varlen_attention_fp32_autograd(q.values, k.values, v.values, q.offsets, causal=causal)
    else:
        out = native.varlen_attention_triton_autograd(q.values, k.values, v.values, q.offsets, causal=causal)
    return Array(values=out, offsets=q.offsets, ragged_dim=0, _host=q._host)


def varlen_rmsnorm(arr: Array, weight=None, eps: float = 1e-6) -> Array:
    """RMSNorm over the last dim of a packed Array."""
    _check_cuda(arr, "varlen_rmsnorm")
    y = native.varlen_rmsnorm_autograd(arr.values, weight, eps)
    return Array(values=y, offsets=arr.offsets, ragged_dim=arr.ragged_dim, _host=arr._host)


def varlen_layernorm(arr: Array, weight=None, bias=None, eps: float = 1e-5) -> Array:
    """LayerNorm over the last dim of a packed Array (biased variance)."""
    _check_cuda(arr, "varlen_layernorm")
    y = native.varlen_layernorm_autograd(arr.values, weight, bias, eps)
    return Array(values=y, offsets=arr.offsets, ragged_dim=arr.ragged_dim, _host=arr._host)


def varlen_softmax(arr: Array) -> Array:
    """Softmax along the ragged dimension, per sequence and feature column."""
    _check_cuda(arr, "varlen_softmax")
    if arr.ragged_dim != 0:
        raise NotImplementedError("varlen_softmax supports ragged_dim=0 only in v0.1")
    y = native.varlen_softmax_packed(arr.values, arr.offsets)
    return Array(values=y, offsets=arr.offsets, ragged_dim=0, _host=arr._host)
