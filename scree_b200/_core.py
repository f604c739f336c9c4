"""scree.Array and its construction ops, with the data movement on the GPU.

Mirrors scree/_core.py (Array :22-94, pack :97-141, unpack :144-158,
to_padded :161-250, from_padded :253-301, from_cu_seqlens :304-309): same
names, argument meanings, return conventions and error types.  The difference
is where the bytes move: pack, to_padded and from_padded run as single
libscree_b200 gather kernels on CUDA tensors (one pass over the data, no
per-row Python loop), and host synchronisation is limited to one small
offsets read where the reference does one per row.

Only CUDA torch tensors are accepted by the data-moving ops; there is no CPU
path.  ``Array`` itself is a plain container and accepts any array type.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, List, Tuple

from . import _lib


def _is_torch(x: Any) -> bool:
    return type(x).__module__.startswith("torch")


def _require_cuda(x: Any, op: str) -> None:
    if not (_is_torch(x) and x.is_cuda):
        raise TypeError(f"scree_b200.{op} requires CUDA torch tensors (got {type(x).__name__})")


def _host_offsets(offsets: Any) -> List[int]:
    """Offsets as Python ints (one device->host copy for CUDA tensors)."""
    if _is_torch(offsets):
        return [int(v) for v in offsets.detach().to("cpu").tolist()]
    return [int(v) for v in list(offsets)]


@dataclass(frozen=True)
class Array:
    """A packed values+offsets array with one variable-length dimension.

    Same contract as scree.Array (scree/_core.py:22-94): ``values`` holds the B
    sequences concatenated along ``ragged_dim``; sequence i occupies
    ``[offsets[i], offsets[i+1])``.  Invariants are checked at construction with
    the reference's messages (scree/_core.py:44-62).
    """

    values: Any
    offsets: Any
    ragged_dim: int = 0
    _host: Any = field(default=None, repr=False, compare=False)

    def __post_init__(self) -> None:
        if self.values.ndim < 1:
            raise ValueError(f"values must be at least 1-D, got {self.values.ndim}-D")
        if not (0 <= self.ragged_dim < self.values.ndim):
            raise ValueError(
                f"ragged_dim={self.ragged_dim} out of range for {self.values.ndim}-D values"
            )
        if self.offsets.ndim != 1:
            raise ValueError(f"offsets must be 1-D, got {self.offsets.ndim}-D")
        if len(self.offsets) < 2:
            raise ValueError("offsets must have length >= 2")
        if self._host is not None:
            first, last = self._host[0], self._host[-1]
        elif _is_torch(self.offsets):
            ends = self.offsets[[0, -1]].tolist()  # one sync for both ends
            first, last = int(ends[0]), int(ends[1])
        else:
            first, last = int(self.offsets[0]), int(self.offsets[-1])
        if first != 0:
            raise ValueError(f"offsets[0] must be 0, got {first}")
        ragged_size = self.values.shape[self.ragged_dim]
        if last != ragged_size:
            raise ValueError(
                f"offsets[-1] ({last}) must equal "
                f"values.shape[ragged_dim={self.ragged_dim}] ({ragged_size})"
            )

    def host_offsets(self) -> List[int]:
        """Offsets as Python ints, cached when the Array was built on the host side."""
        if self._host is not None:
            return list(self._host)
        return _host_offsets(self.offsets)

    @property
    def batch_size(self) -> int:
        return len(self.offsets) - 1

    @property
    def lengths(self) -> Any:
        """Per-row lengths: lengths[i] = offsets[i+1] - offsets[i]."""
        return self.offsets[1:] - self.offsets[:-1]

    @property
    def total_length(self) -> int:
        return int(self.values.shape[self.ragged_dim])

    @property
    def dtype(self) -> Any:
        return self.values.dtype

    @property
    def feature_shape(self) -> tuple:
        return tuple(s for i, s in enumerate(self.values.shape) if i != self.ragged_dim)

    def __len__(self) -> int:
        return self.batch_size

    def __repr__(self) -> str:
        return (
            f"scree.Array(batch_size={self.batch_size}, "
            f"total_length={self.total_length}, "
            f"feature_shape={self.feature_shape}, "
            f"dtype={self.dtype})"
        )


def _pow2_align(addr: int) -> int:
    a = 16
    while a > 1 and addr % a:
        a //= 2
    return a


def pack(arrays: List[Any], ragged_dim: int = 0) -> Array:
    """Pack a list of CUDA tensors into a scree.Array (scree/_core.py:97-141).

    Offsets are int32 of length B+1, as in the reference's torch branch.  The
    concatenation is one gather kernel (scree_pack) over all sources.  Like the
    reference's torch.cat it is differentiable: the gradient of each source is
    its slice of the gradient of ``values``.
    """
    if not arrays:
        raise ValueError("Cannot pack an empty list")
    first = arrays[0]
    _require_cuda(first, "pack")
    dev = first.device
    for a in arrays:
        _require_cuda(a, "pack")
        if a.dtype != first.dtype:
            raise TypeError("all arrays must share a dtype")
        if a.device != dev:
            raise ValueError("all arrays must be on the same device")
        if a.ndim != first.ndim or any(
            a.shape[d] != first.shape[d] for d in range(first.ndim) if d != ragged_dim
        ):
            raise ValueError("all arrays must share the non-ragged dims")
    if ragged_dim != 0:
        # General dim: move the ragged dim first, pack, move it back.
        moved = [a.movedim(ragged_dim, 0) for a in arrays]
        inner = pack(moved, 0)
        values = inner.values.movedim(0, ragged_dim).contiguous()
        return Array(values=values, offsets=inner.offsets, ragged_dim=ragged_dim, _host=inner._host)
    host = [0]
    for a in arrays:
        host.append(host[-1] + int(a.shape[0]))
    if any(a.requires_grad for a in arrays):
        values, offsets = _PackFn.get().apply(tuple(host), *arrays)
    else:
        values, offsets = _pack_values(arrays, host)
    return Array(values=values, offsets=offsets, ragged_dim=0, _host=tuple(host))


def _pack_values(arrays, host):
    import torch

    first = arrays[0]
    dev = first.device
    T = host[-1]
    feat = tuple(first.shape[1:])
    srcs = [a.detach().contiguous() for a in arrays]
    B = len(srcs)
    # One pinned H2D copy carries both the source pointers and the int32 offsets.
    meta = torch.empty(B + (B + 2) // 2 + 1, dtype=torch.int64, pin_memory=True)
    meta[:B] = torch.tensor([s.data_ptr() for s in srcs], dtype=torch.int64)
    meta[B:].view(torch.int32)[: B + 1].copy_(torch.tensor(host, dtype=torch.int32))
    meta_d = meta.to(dev, non_blocking=True)
    ptrs_d = meta_d[:B]
    offsets = meta_d[B:].view(torch.int32)[: B + 1]
    values = torch.empty((T, *feat), dtype=first.dtype, device=dev)
    row_bytes = first.element_size()
    for f in feat:
        row_bytes *= int(f)
    align = 16
    for s in srcs:
        if s.numel():
            align = min(align, _pow2_align(s.data_ptr()))
    if T and row_bytes:
        with torch.cuda.device(dev):
            rc = _lib.load().scree_pack(
                ptrs_d.data_ptr(), offsets.data_ptr(), 0, B, T,
                max(host[i + 1] - host[i] for i in range(B)), row_bytes, align,
                values.data_ptr(), _lib.stream_ptr(dev),
            )
        _lib.check(rc, "scree_pack")
    # Lifetimes: `srcs` and `meta_d` return to torch's caching allocator, which
    # only hands their blocks to later work on this stream; the pinned staging
    # buffer is held by torch's host allocator until its copy has completed.
    return values, offsets


class _PackFn:
    """Lazily built torch.autograd.Function for pack."""

    _fn = None

    @classmethod
    def get(cls):
        if cls._fn is None:
            import torch

            class PackFunction(torch.autograd.Function):
                @staticmethod
                def forward(ctx, host, *arrays):
                    ctx.host = host
                    values, offsets = _pack_values(arrays, list(host))
                    ctx.mark_non_differentiable(offsets)
                    return values, offsets

                @staticmethod
                def backward(ctx, grad_values, _grad_offsets):
                    h = ctx.host
                    return (None, *[grad_values[h[i] : h[i + 1]] for i in range(len(h) - 1)])

            cls._fn = PackFunction
        return cls._fn


def unpack(arr: Array) -> List[Any]:
    """Views of each sequence (scree/_core.py:144-158); one offsets read in total."""
    host = arr.host_offsets()
    rd = arr.ragged_dim
    nd = arr.values.ndim
    out = []
    for i in range(arr.batch_size):
        slc = [slice(None)] * nd
        slc[rd] = slice(host[i], host[i + 1])
        out.append(arr.values[tuple(slc)])
    return out


def _fill_pattern(fill_value: float, dtype) -> bytes:
    import torch

    return torch.tensor([fill_value], dtype=dtype).view(torch.uint8).numpy().tobytes()


def to_padded(arr: Array, side: str = "right", fill_value: float = 0.0) -> Tuple[Any, Any]:
    """Padded (B, max_len, *F) copy plus bool mask (scree/_core.py:161-250).

    One kernel writes every padded element (value or fill) and the mask.
    """
    import torch

    return _to_padded_mask(arr, side, fill_value, torch.bool)


def _to_padded_mask(arr: Array, side: str, fill_value: float, mask_dtype) -> Tuple[Any, Any]:
    """to_padded with the mask written as `mask_dtype` (bool or an integer type)."""
    import torch

    if arr.ragged_dim != 0:
        raise NotImplementedError("to_padded supports ragged_dim=0 only in v0.1")
    if side not in ("right", "left"):
        raise ValueError(f"side must be 'right' or 'left', got {side!r}")
    _require_cuda(arr.values, "to_padded")
    host = arr.host_offsets()
    B = arr.batch_size
    lengths = [host[i + 1] - host[i] for i in range(B)]
    max_len = max(lengths) if lengths else 0
    vals = arr.values.contiguous()
    feat = tuple(vals.shape[1:])
    dev = vals.device
    padded = torch.empty((B, max_len, *feat), dtype=vals.dtype, device=dev)
    mask = torch.empty((B, max_len), dtype=mask_dtype, device=dev)
    offs = arr.offsets
    if not (_is_torch(offs) and offs.device == dev):
        offs = torch.as_tensor(host, dtype=torch.int64, device=dev)
    offs = offs.contiguous()
    row_bytes = vals.element_size()
    for f in feat:
        row_bytes *= int(f)
    pat = _fill_pattern(fill_value, vals.dtype)
    buf = ctypes_buffer(pat)
    if B and max_len:
        with torch.cuda.device(dev):
            rc = _lib.load().scree_to_padded_ex(
                vals.data_ptr(), offs.data_ptr(), 1 if offs.dtype == torch.int64 else 0,
                B, max_len, row_bytes, vals.element_size(), buf, 1 if side == "left" else 0,
                padded.data_ptr(), mask.data_ptr(), mask.element_size(), _lib.stream_ptr(dev),
            )
        _lib.check(rc, "scree_to_padded")
    return padded, mask


def ctypes_buffer(b: bytes):
    import ctypes

    return ctypes.cast(ctypes.create_string_buffer(b, len(b)), ctypes.c_void_p)


def from_padded(padded: Any, mask: Any) -> Array:
    """Packed Array from (padded, mask), right padding assumed (scree/_core.py:253-301).

    Lengths are mask row sums (as in the reference); offsets int32.
    """
    import torch

    _require_cuda(padded, "from_padded")
    return _from_padded_mask(padded, mask.to(device=padded.device, dtype=torch.bool).contiguous())


def _from_padded_mask(padded: Any, m: Any) -> Array:
    """from_padded with a contiguous device mask of bool or 1/2/4/8-byte
    integers (nonzero = valid), read in its own width."""
    import torch

    B = int(padded.shape[0])
    max_len = int(padded.shape[1]) if padded.ndim > 1 else 0
    dev = padded.device
    pad = padded.contiguous()
    offsets = torch.empty(B + 1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        if B == 0:
            offsets.zero_()
        else:
            _lib.check(
                lib.scree_padded_lengths_ex(m.data_ptr(), m.element_size(), B, max_len, offsets.data_ptr(),
                                            _lib.stream_ptr(dev)),
                "scree_padded_lengths",
            )
        host = [int(v) for v in offsets.tolist()]  # the one sync: T sizes the output
        T = host[-1]
        feat = tuple(pad.shape[2:])
        values = torch.empty((T, *feat), dtype=pad.dtype, device=dev)
        row_bytes = pad.element_size()
        for f in feat:
            row_bytes *= int(f)
        if T and row_bytes:
            _lib.check(
                lib.scree_from_padded(pad.data_ptr(), offsets.data_ptr(), B, max_len, T, row_bytes,
                                      values.data_ptr(), _lib.stream_ptr(dev)),
                "scree_from_padded",
            )
    return Array(values=values, offsets=offsets, ragged_dim=0, _host=tuple(host))


def from_cu_seqlens(values: Any, cu_seqlens: Any) -> Array:
    """Zero-copy wrap of FlashAttention's cu_seqlens (scree/_core.py:304-309)."""
    return Array(values=values, offsets=cu_seqlens, ragged_dim=0)
