"""Tensor-level GPU entry points with scree.kernels.triton's names and signatures.

Drop-in for scree/kernels/triton/__init__.py:17-28:
  varlen_attention_triton           scree/kernels/triton/varlen_attention.py:165-268
  varlen_attention_triton_backward  scree/kernels/triton/_backward.py:288-396
  varlen_attention_triton_autograd  scree/kernels/triton/_autograd.py:51-72
  varlen_rmsnorm_triton             scree/kernels/triton/varlen_rmsnorm.py:49-99
  varlen_layernorm_triton           scree/kernels/triton/varlen_layernorm.py:52-109
plus the norm backward passes and autograd wrappers the reference lacks.

All of them call libscree_b200 (hand-written sm_100a kernels) on torch's current
CUDA stream.  Argument checks raise AssertionError with the reference's
messages.  ``block_m`` / ``block_n`` are accepted for signature compatibility;
the tile shape is fixed by head_dim (128 x 128 query x key tiles).  Nothing
here synchronises with the device.
"""

from __future__ import annotations

import math

import torch

from .. import _lib

__all__ = [
    "varlen_attention_triton",
    "varlen_attention_triton_backward",
    "varlen_attention_triton_autograd",
    "varlen_rmsnorm_triton",
    "varlen_layernorm_triton",
    "varlen_rmsnorm_backward",
    "varlen_layernorm_backward",
    "varlen_rmsnorm_autograd",
    "varlen_layernorm_autograd",
    "varlen_softmax_packed",
    "varlen_attention_fp32",
    "varlen_attention_fp32_backward",
    "varlen_attention_fp32_autograd",
    "rmsnorm_qkv",
    "rmsnorm_qkv_autograd",
]


def _offsets_arg(cu_seqlens: torch.Tensor, device) -> tuple[torch.Tensor, int]:
    assert cu_seqlens.ndim == 1 and cu_seqlens.numel() >= 2, "cu_seqlens must be 1-D with >= 2 entries"
    assert cu_seqlens.dtype in (torch.int32, torch.int64), "cu_seqlens must be int32 or int64"
    assert cu_seqlens.device == device, "cu_seqlens must be on the same device as q"
    cu = cu_seqlens.contiguous()
    return cu, 1 if cu.dtype == torch.int64 else 0


def _check_qkv_shapes(q, k, v):
    assert k.shape == v.shape, "k and v must have identical shape"
    assert q.ndim == 3 and q.shape[0] == k.shape[0] and q.shape[2] == k.shape[2], \
        "q, k, v must have identical shape (up to grouped K/V heads)"
    assert k.shape[1] >= 1 and q.shape[1] % k.shape[1] == 0, \
        "the query head count must be a multiple of the K/V head count"


def _attn_view(t: torch.Tensor) -> torch.Tensor:
    """A (T, H, D) view the TMA tensor maps accept: unit inner stride, 16-byte
    aligned base and row/head strides that are multiples of 8 elements."""
    ok = (
        t.stride(2) == 1
        and t.stride(0) % 8 == 0
        and t.stride(1) % 8 == 0
        and t.data_ptr() % 16 == 0
    )
    return t if ok else t.contiguous()


def varlen_attention_triton(
    q,
    k,
    v,
    cu_seqlens,
    causal: bool = False,
    block_m: int = 64,
    block_n: int = 64,
    return_lse: bool = False,
    out=None,
    lse_buffer=None,
    max_seqlen=None,
):
    """Variable-length self-attention forward (scree/kernels/triton/varlen_attention.py:165).

    q, k, v: (total_tokens, n_heads, head_dim) fp16/bf16 CUDA tensors, head_dim in
    {32, 64, 128}.  cu_seqlens: (batch+1,) int32 or int64 offsets.  Returns ``out``
    or ``(out, lse)`` with lse (total_tokens, n_heads) fp32 in natural log.
    ``max_seqlen`` is optional and unused (no host synchronisation is needed).
    Grouped-query attention: k and v may have fewer heads than q (a divisor of
    q's head count); query head h then reads K / V head h // (n_heads / kv_heads).
    """
    _check_qkv_shapes(q, k, v)
    assert q.is_cuda, "varlen_attention_triton requires CUDA tensors"
    assert q.dtype in (torch.float16, torch.bfloat16), "fp16 or bf16 only in v0.0"
    assert k.dtype == q.dtype and v.dtype == q.dtype, "q, k, v must share a dtype"
    total, n_heads, head_dim = q.shape
    cu, is64 = _offsets_arg(cu_seqlens, q.device)
    batch = cu.numel() - 1
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    else:
        assert out.shape == q.shape and out.dtype == q.dtype and out.device == q.device
    if lse_buffer is None:
        lse = torch.empty((total, n_heads), dtype=torch.float32, device=q.device)
    else:
        assert lse_buffer.shape == (total, n_heads)
        assert lse_buffer.dtype == torch.float32 and lse_buffer.device == q.device
        assert lse_buffer.is_contiguous(), "lse_buffer must be contiguous"
        lse = lse_buffer
    if total == 0:
        return (out, lse) if return_lse else out
    qv, kv, vv = _attn_view(q), _attn_view(k), _attn_view(v)
    kv_heads = k.shape[1]
    o_direct = out.stride(2) == 1 and out.stride(0) % 8 == 0 and out.stride(1) % 8 == 0 and out.data_ptr() % 16 == 0
    o_buf = out if o_direct else torch.empty_like(q, memory_format=torch.contiguous_format)
    lib = _lib.load()
    ws = torch.empty(lib.scree_attn_fwd_workspace_size(batch, total, n_heads, head_dim), dtype=torch.uint8, device=q.device)
    scale = 1.0 / math.sqrt(head_dim)
    with torch.cuda.device(q.device):
        rc = lib.scree_attn_fwd_gqa(
            qv.data_ptr(), kv.data_ptr(), vv.data_ptr(),
            qv.stride(0), qv.stride(1), kv.stride(0), kv.stride(1), vv.stride(0), vv.stride(1),
            cu.data_ptr(), is64, batch, total, n_heads, kv_heads, head_dim, _lib.dtype_code(q.dtype),
            1 if causal else 0, scale, int(max_seqlen or 0),
            o_buf.data_ptr(), o_buf.stride(0), o_buf.stride(1), lse.data_ptr(),
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "varlen_attention_triton")
    if not o_direct:
        out.copy_(o_buf)
    return (out, lse) if return_lse else out


def varlen_attention_triton_backward(
    do, q, k, v, o, lse, cu_seqlens, causal: bool = False, block_m: int = 64, block_n: int = 64
):
    """dq, dk, dv of varlen self-attention (scree/kernels/triton/_backward.py:288).

    One sm_100a kernel computes all three gradients per 128-key tile (five GEMMs,
    none recomputed), after a Delta = rowsum(O * dO) pass; dq is accumulated in
    fp32 and cast once at the end.  With grouped-query k / v (fewer heads), dk
    and dv have k's shape and sum over the query heads sharing each K / V head.
    """
    _check_qkv_shapes(q, k, v)
    assert q.shape == o.shape == do.shape, "shape mismatch"
    assert q.is_cuda, "varlen_attention_triton_backward requires CUDA tensors"
    assert q.dtype in (torch.float16, torch.bfloat16), "fp16 or bf16 only in v0.0"
    total, n_heads, head_dim = q.shape
    assert lse.shape == (total, n_heads) and lse.dtype == torch.float32
    cu, is64 = _offsets_arg(cu_seqlens, q.device)
    batch = cu.numel() - 1
    q, k, v, o, do = (t.contiguous() for t in (q, k, v, o, do))
    lse = lse.contiguous()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    if total == 0:
        return dq, dk, dv
    lib = _lib.load()
    ws = torch.empty(lib.scree_attn_bwd_workspace_size(batch, total, n_heads, head_dim), dtype=torch.uint8, device=q.device)
    scale = 1.0 / math.sqrt(head_dim)
    with torch.cuda.device(q.device):
        rc = lib.scree_attn_bwd_gqa(
            do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
            cu.data_ptr(), is64, batch, total, n_heads, k.shape[1], head_dim, _lib.dtype_code(q.dtype),
            1 if causal else 0, scale, 0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "varlen_attention_triton_backward")
    return dq, dk, dv


class _VarlenAttention(torch.autograd.Function):
    """Forward and backward on the sm_100a kernels (scree/kernels/triton/_autograd.py:24-48)."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, causal):
        out, lse = varlen_attention_triton(q, k, v, cu_seqlens, causal=causal, return_lse=True)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens)
        ctx.causal = causal
        return out

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, out, lse, cu_seqlens = ctx.saved_tensors
        dq, dk, dv = varlen_attention_triton_backward(
            grad_output.contiguous(), q, k, v, out, lse, cu_seqlens, causal=ctx.causal
        )
        return dq, dk, dv, None, None


def varlen_attention_triton_autograd(q, k, v, cu_seqlens, causal: bool = False):
    """Autograd-aware varlen attention (scree/kernels/triton/_autograd.py:51)."""
    return _VarlenAttention.apply(q, k, v, cu_seqlens, causal)


# --------------------------------------------------------------------------- fp32 attention


def varlen_attention_fp32(q, k, v, cu_seqlens, causal: bool = False):
    """fp32 varlen attention forward on CUDA-core fp32 kernels (fp32-grade
    results); returns (out, lse).  The reference's Array-level op computes in the
    caller's dtype, fp32 included (scree/kernels/reference/varlen_attention.py:90-114)."""
    _check_qkv_shapes(q, k, v)
    assert q.is_cuda and q.dtype == torch.float32, "fp32 CUDA tensors expected"
    assert k.dtype == q.dtype and v.dtype == q.dtype, "q, k, v must share a dtype"
    total, n_heads, head_dim = q.shape
    cu, is64 = _offsets_arg(cu_seqlens, q.device)
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    lse = torch.empty((total, n_heads), dtype=torch.float32, device=q.device)
    if total == 0:
        return out, lse
    q, k, v = (t if t.stride(2) == 1 else t.contiguous() for t in (q, k, v))
    with torch.cuda.device(q.device):
        rc = _lib.load().scree_attn_fwd_gqa(
            q.data_ptr(), k.data_ptr(), v.data_ptr(),
            q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
            cu.data_ptr(), is64, cu.numel() - 1, total, n_heads, k.shape[1], head_dim, _lib.F32,
            1 if causal else 0, 1.0 / math.sqrt(head_dim), 0,
            out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), None, 0,
            _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "varlen_attention (fp32)")
    return out, lse


def varlen_attention_fp32_backward(do, q, k, v, o, lse, cu_seqlens, causal: bool = False):
    """(dq, dk, dv) of varlen_attention_fp32, fp32 throughout, deterministic."""
    total, n_heads, head_dim = q.shape
    cu, is64 = _offsets_arg(cu_seqlens, q.device)
    q, k, v, o, do = (t.contiguous() for t in (q, k, v, o, do))
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    if total == 0:
        return dq, dk, dv
    lib = _lib.load()
    ws = torch.empty(lib.scree_attn_bwd_workspace_size(cu.numel() - 1, total, n_heads, head_dim),
                     dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.scree_attn_bwd_gqa(
            do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.contiguous().data_ptr(),
            cu.data_ptr(), is64, cu.numel() - 1, total, n_heads, k.shape[1], head_dim, _lib.F32,
            1 if causal else 0, 1.0 / math.sqrt(head_dim), 0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device),
        )
    _lib.check(rc, "varlen_attention backward (fp32)")
    return dq, dk, dv


class _VarlenAttentionF32(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, causal):
        out, lse = varlen_attention_fp32(q, k, v, cu_seqlens, causal)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens)
        ctx.causal = causal
        return out

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, out, lse, cu_seqlens = ctx.saved_tensors
        dq, dk, dv = varlen_attention_fp32_backward(grad_output, q, k, v, out, lse, cu_seqlens, ctx.causal)
        return dq, dk, dv, None, None


def varlen_attention_fp32_autograd(q, k, v, cu_seqlens, causal: bool = False):
    """Differentiable fp32 varlen attention (forward and backward on fp32 kernels)."""
    return _VarlenAttentionF32.apply(q, k, v, cu_seqlens, causal)


# --------------------------------------------------------------------------- norms


def _norm_prep(x, weight, name):
    assert x.is_cuda, f"{name} requires CUDA tensors"
    assert x.dtype in (torch.float16, torch.bfloat16, torch.float32), "fp16, bf16 or fp32 only"
    feature_dim = x.shape[-1]
    x_flat = x.reshape(-1, feature_dim)
    if x_flat.stride(-1) != 1:
        x_flat = x_flat.contiguous()
    if weight is not None:
        assert weight.shape == (feature_dim,)
        assert weight.device == x.device
        weight = weight.contiguous()
    return x_flat, weight, feature_dim


def _wcode(weight, x):
    return _lib.dtype_code(weight.dtype) if weight is not None else _lib.dtype_code(x.dtype)


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _rmsnorm_fwd(x, weight, eps, want_stats):
    x_flat, weight, C = _norm_prep(x, weight, "varlen_rmsnorm_triton")
    rows = x_flat.shape[0]
    y = torch.empty((rows, C), dtype=x.dtype, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device) if want_stats else None
    with torch.cuda.device(x.device):
        rc = _lib.load().scree_rmsnorm_fwd(
            x_flat.data_ptr(), x_flat.stride(0), _ptr(weight), _wcode(weight, x), y.data_ptr(), C,
            _ptr(rstd), rows, C, _lib.dtype_code(x.dtype), float(eps), _lib.stream_ptr(x.device),
        )
    _lib.check(rc, "varlen_rmsnorm_triton")
    return y.reshape(x.shape), rstd


def _layernorm_fwd(x, weight, bias, eps, want_stats):
    x_flat, weight, C = _norm_prep(x, weight, "varlen_layernorm_triton")
    if bias is not None:
        assert bias.shape == (C,) and bias.device == x.device
        bias = bias.contiguous()
        if weight is not None:
            assert bias.dtype == weight.dtype, "weight and bias must share a dtype"
    rows = x_flat.shape[0]
    y = torch.empty((rows, C), dtype=x.dtype, device=x.device)
    mean = torch.empty(rows, dtype=torch.float32, device=x.device) if want_stats else None
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device) if want_stats else None
    wref = weight if weight is not None else bias
    with torch.cuda.device(x.device):
        rc = _lib.load().scree_layernorm_fwd(
            x_flat.data_ptr(), x_flat.stride(0), _ptr(weight), _ptr(bias), _wcode(wref, x),
            y.data_ptr(), C, _ptr(mean), _ptr(rstd), rows, C, _lib.dtype_code(x.dtype), float(eps),
            _lib.stream_ptr(x.device),
        )
    _lib.check(rc, "varlen_layernorm_triton")
    return y.reshape(x.shape), mean, rstd


def varlen_rmsnorm_triton(x, weight=None, eps: float = 1e-6):
    """RMSNorm over the last dim (scree/kernels/triton/varlen_rmsnorm.py:49).

    Statistics in fp32; the weight is applied in its own dtype (the oracle's
    numerics, reference/varlen_rmsnorm.py:58-65).  Same shape/dtype as x.
    """
    return _rmsnorm_fwd(x, weight, eps, False)[0]


def varlen_layernorm_triton(x, weight=None, bias=None, eps: float = 1e-5):
    """LayerNorm over the last dim, biased variance (scree/kernels/triton/varlen_layernorm.py:52)."""
    return _layernorm_fwd(x, weight, bias, eps, False)[0]


def _norm_bwd_ws(rows, C, device):
    n = _lib.load().scree_norm_bwd_workspace_size(rows, C)
    return torch.empty(n, dtype=torch.uint8, device=device)


def varlen_rmsnorm_backward(dy, x, weight, rstd):
    """(dx, dweight or None) for y = rmsnorm(x) * weight, from the saved rstd."""
    C = x.shape[-1]
    x_flat = x.reshape(-1, C).contiguous()
    dy_flat = dy.reshape(-1, C).contiguous()
    rows = x_flat.shape[0]
    dx = torch.empty_like(x_flat)
    dw = torch.empty(C, dtype=torch.float32, device=x.device) if weight is not None else None
    ws = _norm_bwd_ws(rows, C, x.device) if dw is not None else None
    with torch.cuda.device(x.device):
        rc = _lib.load().scree_rmsnorm_bwd(
            dy_flat.data_ptr(), x_flat.data_ptr(), _ptr(weight), _wcode(weight, x), rstd.data_ptr(),
            dx.data_ptr(), _ptr(dw), rows, C, _lib.dtype_code(x.dtype), _ptr(ws),
            ws.numel() if ws is not None else 0, _lib.stream_ptr(x.device),
        )
    _lib.check(rc, "varlen_rmsnorm_backward")
    return dx.reshape(x.shape), (dw.to(weight.dtype) if dw is not None else None)


def varlen_layernorm_backward(dy, x, weight, bias, mean, rstd):
    """(dx, dweight or None, dbias or None) for y = layernorm(x) * weight + bias."""
    C = x.shape[-1]
    x_flat = x.reshape(-1, C).contiguous()
    dy_flat = dy.reshape(-1, C).contiguous()
    rows = x_flat.shape[0]
    dx = torch.empty_like(x_flat)
    dw = torch.empty(C, dtype=torch.float32, device=x.device) if weight is not None else None
    db = torch.empty(C, dtype=torch.float32, device=x.device) if bias is not None else None
    ws = _norm_bwd_ws(rows, C, x.device) if (dw is not None or db is not None) else None
    wref = weight if weight is not None else bias
    with torch.cuda.device(x.device):
        rc = _lib.load().scree_layernorm_bwd(
            dy_flat.data_ptr(), x_flat.data_ptr(), _ptr(weight), _wcode(wref, x), mean.data_ptr(),
            rstd.data_ptr(), dx.data_ptr(), _ptr(dw), _ptr(db), rows, C, _lib.dtype_code(x.dtype),
            _ptr(ws), ws.numel() if ws is not None else 0, _lib.stream_ptr(x.device),
        )
    _lib.check(rc, "varlen_layernorm_backward")
    return (
        dx.reshape(x.shape),
        dw.to(weight.dtype) if dw is not None else None,
        db.to(bias.dtype) if db is not None else None,
    )


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        y, rstd = _rmsnorm_fwd(x, weight, eps, True)
        ctx.save_for_backward(x, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        dx, dw = varlen_rmsnorm_backward(dy, x, weight, rstd)
        if weight is None or not ctx.needs_input_grad[1]:
            dw = None
        return dx, dw, None


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        y, mean, rstd = _layernorm_fwd(x, weight, bias, eps, True)
        ctx.save_for_backward(x, weight, bias, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, bias, mean, rstd = ctx.saved_tensors
        dx, dw, db = varlen_layernorm_backward(dy, x, weight, bias, mean, rstd)
        return dx, (dw if ctx.needs_input_grad[1] else None), (db if ctx.needs_input_grad[2] else None), None


def varlen_rmsnorm_autograd(x, weight=None, eps: float = 1e-6):
    """Differentiable varlen RMSNorm (forward and backward on sm_100a kernels)."""
    return _RMSNorm.apply(x, weight, eps)


def varlen_layernorm_autograd(x, weight=None, bias=None, eps: float = 1e-5):
    """Differentiable varlen LayerNorm (forward and backward on sm_100a kernels)."""
    return _LayerNorm.apply(x, weight, bias, eps)


# --------------------------------------------------------------------------- softmax


def _softmax_call(fn, what, offs, out, *tensors):
    cu, is64 = _offsets_arg(offs, tensors[0].device)
    T = tensors[0].shape[0]
    F = 1
    for d in tensors[0].shape[1:]:
        F *= int(d)
    with torch.cuda.device(tensors[0].device):
        rc = fn(*[t.data_ptr() for t in tensors], cu.data_ptr(), is64, cu.numel() - 1, T, F,
                _lib.dtype_code(tensors[0].dtype), out.data_ptr(), _lib.stream_ptr(tensors[0].device))
    _lib.check(rc, what)


class _VarlenSoftmax(torch.autograd.Function):
    @staticmethod
    def forward(ctx, values, offsets):
        x = values.contiguous()
        y = torch.empty_like(x)
        _softmax_call(_lib.load().scree_softmax_fwd, "varlen_softmax", offsets, y, x)
        ctx.save_for_backward(y, offsets)
        return y

    @staticmethod
    def backward(ctx, dy):
        y, offsets = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch.empty_like(y)
        _softmax_call(_lib.load().scree_softmax_bwd, "varlen_softmax backward", offsets, dx, dy, y)
        return dx, None


def varlen_softmax_packed(values, offsets):
    """Softmax along the ragged (first) dim of packed (T, ...) values within each
    sequence [offsets[b], offsets[b+1]), per feature column; differentiable.
    Tensor-level form of scree/kernels/reference/varlen_softmax.py:13."""
    assert values.is_cuda, "varlen_softmax requires CUDA tensors"
    assert values.dtype in (torch.float16, torch.bfloat16, torch.float32), "fp16, bf16 or fp32 only"
    return _VarlenSoftmax.apply(values, offsets)


# --------------------------------------------------------------------------- fused pre-norm QKV


def rmsnorm_qkv(x, gamma, weight, eps: float = 1e-6, want_rstd: bool = False):
    """``(rmsnorm(x) * gamma) @ weight`` in one tcgen05 GEMM with the RMSNorm fused
    into it (the caller-side sequence of scree/examples/03_train_step.py:36-41).

    x: (T, C) fp16 / bf16 CUDA tensor (any row stride that is a multiple of 8);
    gamma: (C,) or None; weight: (C, N) in x's dtype, N a multiple of 128 and C of
    64.  Returns y (T, N) in x's dtype (view it as (T, 3, H, D) for attention),
    and rstd (T,) fp32 when ``want_rstd``."""
    assert x.is_cuda and x.ndim == 2 and x.dtype in (torch.float16, torch.bfloat16)
    assert weight.ndim == 2 and weight.shape[0] == x.shape[1] and weight.dtype == x.dtype
    T, C = x.shape
    N = weight.shape[1]
    if x.stride(1) != 1 or x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        x = x.contiguous()
    weight = weight.contiguous()
    y = torch.empty((T, N), dtype=x.dtype, device=x.device)
    rstd = torch.empty(T, dtype=torch.float32, device=x.device) if want_rstd else None
    lib = _lib.load()
    if gamma is not None:
        assert gamma.shape == (C,) and gamma.device == x.device
        gamma = gamma.contiguous()
    ws = torch.empty(lib.scree_rmsnorm_qkv_workspace_size(T, C, N), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        rc = lib.scree_rmsnorm_qkv_fwd(
            x.data_ptr(), x.stride(0), _ptr(gamma), _wcode(gamma, x), weight.data_ptr(), y.data_ptr(),
            _ptr(rstd), T, C, N, _lib.dtype_code(x.dtype), float(eps), ws.data_ptr(), ws.numel(),
            _lib.stream_ptr(x.device),
        )
    _lib.check(rc, "rmsnorm_qkv")
    return (y, rstd) if want_rstd else y


class _RMSNormQKV(torch.autograd.Function):
    """Forward: the fused kernel.  Backward: h = rmsnorm(x) * gamma recomputed by
    the RMSNorm kernel, dH = dY W^T and dW = h^T dY as library GEMMs, then dx and
    dgamma from the RMSNorm backward kernel."""

    @staticmethod
    def forward(ctx, x, gamma, weight, eps):
        y, rstd = rmsnorm_qkv(x, gamma, weight, eps, want_rstd=True)
        ctx.save_for_backward(x, gamma, weight, rstd)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gamma, weight, rstd = ctx.saved_tensors
        h = varlen_rmsnorm_triton(x, gamma, ctx.eps)
        dy = dy.contiguous()
        dh = dy @ weight.t()
        dw = h.t() @ dy if ctx.needs_input_grad[2] else None
        dx, dg = varlen_rmsnorm_backward(dh, x, gamma, rstd)
        return dx, (dg if gamma is not None and ctx.needs_input_grad[1] else None), dw, None


def rmsnorm_qkv_autograd(x, gamma, weight, eps: float = 1e-6):
    """Differentiable rmsnorm_qkv."""
    return _RMSNormQKV.apply(x, gamma, weight, eps)
