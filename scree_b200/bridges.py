"""Bridges between scree_b200.Array and the varlen formats either side of the
hot path, with the data movement on the GPU.

Same names, arguments and conventions as scree/bridges (scree/bridges/__init__.py:14-25):

  from_hf_padded(hidden_states, attention_mask) -> Array   _hf_padded.py:15-29
  to_hf_padded(arr) -> (hidden_states, attention_mask)     _hf_padded.py:32-46
  to_torch_nested(arr) -> jagged NestedTensor              _torch_nested.py:10-22
  from_torch_nested(nt) -> Array                           _torch_nested.py:25-47
  to_torch(arr) / to_numpy(arr)                            _dlpack.py:10-41

The HF bridges run the libscree_b200 gather kernels: the attention mask is
read in its own integer width (HF passes int64) by the lengths kernel, and
to_hf_padded writes the int64 mask directly from the to_padded kernel, so
neither direction makes a separate mask-conversion pass.  to_torch_nested
wraps the packed buffer and its offsets as a jagged NestedTensor without
copying (the reference copies every row through torch.nested.nested_tensor).
"""

from __future__ import annotations

from typing import Any, Tuple

from . import _core, _lib
from ._core import Array, _is_torch

__all__ = ["to_torch_nested", "from_torch_nested", "to_hf_padded", "from_hf_padded", "to_torch", "to_numpy"]


def from_hf_padded(hidden_states: Any, attention_mask: Any) -> Array:
    """HF ``(hidden_states (B, S, *F), attention_mask (B, S))`` -> packed Array.

    Right padding (HF convention: 1 marks a real token, 0 padding); lengths are
    the mask row sums, as in the reference (which goes through from_padded).
    Any integer or bool mask dtype is read as is on the device."""
    import torch

    _core._require_cuda(hidden_states, "from_hf_padded")
    mask = attention_mask
    if not _is_torch(mask):
        mask = torch.as_tensor(mask)
    mask = mask.to(device=hidden_states.device)
    if mask.dtype == torch.bool or mask.element_size() not in (1, 2, 4, 8) or mask.is_floating_point():
        mask = mask.to(torch.bool)
    return _core._from_padded_mask(hidden_states, mask.contiguous())


def to_hf_padded(arr: Array) -> Tuple[Any, Any]:
    """Packed Array -> HF ``(hidden_states, attention_mask)``: right padding with
    zeros, attention_mask int64 (1 valid, 0 padding)."""
    import torch

    return _core._to_padded_mask(arr, side="right", fill_value=0.0, mask_dtype=torch.int64)


def to_torch_nested(arr: Array) -> Any:
    """Packed Array -> torch jagged NestedTensor over the same storage (no copy)."""
    import torch

    if arr.ragged_dim != 0:
        raise NotImplementedError("to_torch_nested supports ragged_dim=0 only")
    offs = arr.offsets
    if not _is_torch(offs):
        offs = torch.as_tensor(offs)
    offs = offs.to(device=arr.values.device, dtype=torch.int64)
    return torch.nested.nested_tensor_from_jagged(arr.values, offs)


def from_torch_nested(nt: Any) -> Array:
    """Jagged NestedTensor -> packed Array over its values and offsets (no copy)."""
    if not getattr(nt, "is_nested", False):
        raise TypeError(f"expected a NestedTensor, got {type(nt).__name__}")
    import torch

    try:
        values = nt.values()
        offsets = nt.offsets().to(torch.int32)
    except (AttributeError, RuntimeError):
        rows = list(nt.unbind())
        return _core.pack(rows)
    return Array(values=values, offsets=offsets, ragged_dim=0)


def to_torch(arr: Array) -> Array:
    """Array with torch values / offsets (zero-copy from numpy; unchanged if already torch)."""
    import torch

    if _is_torch(arr.values):
        return arr
    values = torch.from_numpy(arr.values) if hasattr(arr.values, "__array__") else torch.from_dlpack(arr.values)
    offsets = torch.from_numpy(arr.offsets) if hasattr(arr.offsets, "__array__") else torch.from_dlpack(arr.offsets)
    return Array(values=values, offsets=offsets.to(torch.int32), ragged_dim=arr.ragged_dim)


def to_numpy(arr: Array) -> Array:
    """Array with numpy values / offsets (copies device tensors to the host)."""
    import numpy as np

    if not _is_torch(arr.values):
        return arr
    values = arr.values.detach().cpu().numpy()
    offsets = arr.offsets.detach().cpu().numpy()
    return Array(values=values, offsets=offsets.astype(np.int32), ragged_dim=arr.ragged_dim)


