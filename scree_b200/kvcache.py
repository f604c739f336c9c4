"""KV-cache support for inference (the reference lists it as planned,
docs/kernels.md:176-179): appending new tokens' K / V to each sequence's cached
rows, and attention of new queries against the cached + new keys.

  kv_append(cache, new) -> Array              one gather kernel (scree_kv_append)
  varlen_attention_kv(q, k, v, causal=True)   q Array (new tokens), k / v Arrays
                                              (cache + new), offsets of their own
Causal masking is aligned at the end of each sequence: query i of Lq new
queries sees keys j <= i + (Lk - Lq), so decode (Lq = 1) sees the whole cache
and a chunk of prefill sees the cache plus its own earlier tokens.  Forward
only (inference); fp16 / bf16, head_dim 32 / 64 / 128, grouped K/V heads.
"""

from __future__ import annotations

import math

from . import _lib
from ._core import Array, _require_cuda


def _dev_offsets(arr: Array):
    import torch

    offs = arr.offsets
    if not (hasattr(offs, "is_cuda") and offs.is_cuda and offs.device == arr.values.device):
        offs = torch.as_tensor(arr.host_offsets(), dtype=torch.int64, device=arr.values.device)
    return offs.to(torch.int64).contiguous()


def kv_append(cache: Array, new: Array) -> Array:
    """Per sequence, cache rows then new rows, in one packed Array (int64 offsets)."""
    import torch

    _require_cuda(cache.values, "kv_append")
    _require_cuda(new.values, "kv_append")
    if cache.batch_size != new.batch_size:
        raise ValueError(f"batch sizes differ: {cache.batch_size} vs {new.batch_size}")
    if tuple(cache.values.shape[1:]) != tuple(new.values.shape[1:]) or cache.values.dtype != new.values.dtype:
        raise ValueError("cache and new rows must share feature shape and dtype")
    hc, hn = cache.host_offsets(), new.host_offsets()
    B = cache.batch_size
    host = [hc[i] + hn[i] for i in range(B + 1)]
    dev = cache.values.device
    cv, nv = cache.values.contiguous(), new.values.contiguous()
    out = torch.empty((host[-1], *cv.shape[1:]), dtype=cv.dtype, device=dev)
    out_offs = torch.empty(B + 1, dtype=torch.int64, device=dev)
    row_bytes = cv.element_size()
    for f in cv.shape[1:]:
        row_bytes *= int(f)
    max_rows = max((host[i + 1] - host[i] for i in range(B)), default=0)
    with torch.cuda.device(dev):
        rc = _lib.load().scree_kv_append(
            cv.data_ptr(), _dev_offsets(cache).data_ptr(), nv.data_ptr(), _dev_offsets(new).data_ptr(), 1,
            B, cv.shape[0], nv.shape[0], max_rows, row_bytes, out.data_ptr(), out_offs.data_ptr(),
            _lib.stream_ptr(dev),
        )
    _lib.check(rc, "scree_kv_append")
    return Array(values=out, offsets=out_offs, ragged_dim=0, _host=tuple(host))


def varlen_attention_kv(q: Array, k: Array, v: Array, causal: bool = True, return_lse: bool = False):
    """Attention of q's rows against k / v rows with their own offsets (same
    batch), scale 1/sqrt(head_dim); returns an Array on q's offsets (and the LSE
    (Tq, H) fp32 when ``return_lse``)."""
    import torch

    for a in (q, k, v):
        _require_cuda(a.values, "varlen_attention_kv")
    if not (q.batch_size == k.batch_size == v.batch_size):
        raise ValueError("q, k, v must have the same batch size")
    qt, kt, vt = q.values, k.values, v.values
    assert qt.dtype in (torch.float16, torch.bfloat16), "fp16 or bf16 only"
    assert kt.shape == vt.shape and kt.dtype == qt.dtype == vt.dtype
    assert qt.ndim == 3 and qt.shape[2] == kt.shape[2] and qt.shape[1] % kt.shape[1] == 0
    Tq, H, D = qt.shape
    Tk, Hkv = kt.shape[0], kt.shape[1]
    qt, kt, vt = (t if (t.stride(2) == 1 and t.stride(0) % 8 == 0 and t.stride(1) % 8 == 0
                        and t.data_ptr() % 16 == 0) else t.contiguous() for t in (qt, kt, vt))
    out = torch.empty((Tq, H, D), dtype=qt.dtype, device=qt.device)
    lse = torch.empty((Tq, H), dtype=torch.float32, device=qt.device)
    B = q.batch_size
    if Tq:
        lib = _lib.load()
        ws = torch.empty(lib.scree_attn_fwd_workspace_size(B, Tq, H, D), dtype=torch.uint8, device=qt.device)
        with torch.cuda.device(qt.device):
            rc = lib.scree_attn_fwd_kv(
                qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), qt.stride(0), qt.stride(1), kt.stride(0),
                kt.stride(1), vt.stride(0), vt.stride(1), _dev_offsets(q).data_ptr(), _dev_offsets(k).data_ptr(),
                1, B, Tq, Tk, H, Hkv, D, _lib.dtype_code(qt.dtype), 1 if causal else 0, 1.0 / math.sqrt(D),
                out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), ws.data_ptr(), ws.numel(),
                _lib.stream_ptr(qt.device),
            )
        _lib.check(rc, "varlen_attention_kv")
    res = Array(values=out, offsets=q.offsets, ragged_dim=0, _host=q._host)
    return (res, lse) if return_lse else res
