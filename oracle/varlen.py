"""numpy restatement of scree's varlen reference path (test oracle only).

Forward functions follow the reference's numpy branches line by line in
meaning; backward functions are the analytic gradients of those forward
formulas (the reference has no explicit backward: its torch branch is
differentiated by autograd, tests/test_autograd.py:28-64), and they are pinned
against torch autograd through the reference in tests/golden.

All math is done in float64 unless the caller passes something else through
``dtype``; inputs are upcast first.
"""

from __future__ import annotations

import math
from typing import List, Sequence, Tuple

import numpy as np


# --------------------------------------------------------------------------- gathers
def pack(arrays: Sequence[np.ndarray]) -> Tuple[np.ndarray, np.ndarray]:
    """Concatenate along axis 0; int32 offsets with a leading 0.

    Follows src/scree/_core.py:133-139 (numpy branch of pack).
    """
    if len(arrays) == 0:
        raise ValueError("Cannot pack an empty list")
    offsets = np.zeros(len(arrays) + 1, dtype=np.int32)
    offsets[1:] = np.cumsum([a.shape[0] for a in arrays])
    return np.concatenate(arrays, axis=0), offsets


def unpack(values: np.ndarray, offsets: np.ndarray) -> List[np.ndarray]:
    """Slices [offsets[i], offsets[i+1]) (src/scree/_core.py:144-158)."""
    return [values[int(offsets[i]) : int(offsets[i + 1])] for i in range(len(offsets) - 1)]


def to_padded(values: np.ndarray, offsets: np.ndarray, side: str = "right", fill_value=0.0):
    """(B, max_len, *F) padded array and bool mask (src/scree/_core.py:171-250)."""
    if side not in ("right", "left"):
        raise ValueError(f"side must be 'right' or 'left', got {side!r}")
    B = len(offsets) - 1
    lengths = [int(offsets[i + 1] - offsets[i]) for i in range(B)]
    max_len = max(lengths) if lengths else 0
    padded = np.full((B, max_len, *values.shape[1:]), fill_value, dtype=values.dtype)
    mask = np.zeros((B, max_len), dtype=np.bool_)
    for i, n in enumerate(lengths):
        row = values[int(offsets[i]) : int(offsets[i]) + n]
        if side == "right":
            padded[i, :n] = row
            mask[i, :n] = True
        else:
            padded[i, max_len - n :] = row
            mask[i, max_len - n :] = True
    return padded, mask


def from_padded(padded: np.ndarray, mask: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Inverse of right padding; lengths are mask row sums (src/scree/_core.py:291-299)."""
    B = padded.shape[0]
    lengths = [int(mask[i].sum()) for i in range(B)]
    rows = [padded[i, : lengths[i]] for i in range(B)]
    offsets = np.zeros(B + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(lengths)
    if rows:
        values = np.concatenate(rows, axis=0)
    else:
        values = np.zeros((0, *padded.shape[2:]), dtype=padded.dtype)
    return values, offsets


# --------------------------------------------------------------------------- attention
def _seq_scores(qi, ki, scale, causal):
    """(H, L, L) scores of one sequence; einsum("ihd,jhd->hij") of the reference
    written as a batched matmul so long sequences stay fast."""
    s = np.matmul(qi.transpose(1, 0, 2), ki.transpose(1, 2, 0)) * scale
    if causal:
        L = qi.shape[0]
        s = np.where(np.triu(np.ones((L, L), dtype=bool), k=1), -np.inf, s)
    return s


def attention_fwd(q, k, v, offsets, causal=False, scale=None, dtype=np.float64):
    """Per-sequence softmax attention; returns (out (T,H,D), lse (T,H)).

    Follows src/scree/kernels/reference/varlen_attention.py:115-138 (numpy
    branch): scores = q k^T * 1/sqrt(D), triu(k=1) causal mask to -inf, softmax
    with max subtraction, out = attn v.  lse = max + log(sum exp), the quantity
    scree's Triton kernel saves (triton/varlen_attention.py:160).
    """
    q, k, v = (np.asarray(t, dtype=dtype) for t in (q, k, v))
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    T, H, D = q.shape
    out = np.zeros((T, H, D), dtype=dtype)
    lse = np.zeros((T, H), dtype=dtype)
    for i in range(len(offsets) - 1):
        s0, e0 = int(offsets[i]), int(offsets[i + 1])
        if e0 == s0:
            continue
        sc = _seq_scores(q[s0:e0], k[s0:e0], scale, causal)
        m = sc.max(axis=-1, keepdims=True)
        ex = np.exp(sc - m)
        den = ex.sum(axis=-1, keepdims=True)
        attn = ex / den
        out[s0:e0] = np.matmul(attn, v[s0:e0].transpose(1, 0, 2)).transpose(1, 0, 2)
        lse[s0:e0] = (m + np.log(den))[..., 0].T
    return out, lse


def attention_bwd(do, q, k, v, offsets, causal=False, scale=None, dtype=np.float64):
    """Gradients (dq, dk, dv) of attention_fwd's output against upstream do.

    With P = softmax(S), S = scale * Q K^T (masked):
      dV = P^T dO,  dP = dO V^T,  dS = P * (dP - rowsum(dP * P)),
      dQ = scale * dS K,  dK = scale * dS^T Q.
    """
    q, k, v, do = (np.asarray(t, dtype=dtype) for t in (q, k, v, do))
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for i in range(len(offsets) - 1):
        s0, e0 = int(offsets[i]), int(offsets[i + 1])
        if e0 == s0:
            continue
        qh, kh, vh, doh = (t[s0:e0].transpose(1, 0, 2) for t in (q, k, v, do))  # (H, L, D)
        sc = _seq_scores(q[s0:e0], k[s0:e0], scale, causal)
        m = sc.max(axis=-1, keepdims=True)
        ex = np.exp(sc - m)
        P = ex / ex.sum(axis=-1, keepdims=True)  # (H, L, L)
        dv[s0:e0] = np.matmul(P.transpose(0, 2, 1), doh).transpose(1, 0, 2)
        dP = np.matmul(doh, vh.transpose(0, 2, 1))
        dS = P * (dP - (dP * P).sum(axis=-1, keepdims=True))
        dq[s0:e0] = (scale * np.matmul(dS, kh)).transpose(1, 0, 2)
        dk[s0:e0] = (scale * np.matmul(dS.transpose(0, 2, 1), qh)).transpose(1, 0, 2)
    return dq, dk, dv


# --------------------------------------------------------------------------- norms
def rmsnorm_fwd(x, weight=None, eps=1e-6, dtype=np.float64):
    """y = x / sqrt(mean(x^2) + eps) * weight
    (src/scree/kernels/reference/varlen_rmsnorm.py:58-65)."""
    x = np.asarray(x, dtype=dtype)
    rms = np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    y = x / rms
    if weight is not None:
        y = y * np.asarray(weight, dtype=dtype)
    return y


def rmsnorm_bwd(dy, x, weight=None, eps=1e-6, dtype=np.float64):
    """(dx, dweight) of rmsnorm_fwd; dweight None when weight is None."""
    x = np.asarray(x, dtype=dtype)
    dy = np.asarray(dy, dtype=dtype)
    C = x.shape[-1]
    r = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    xh = x * r
    g = dy * np.asarray(weight, dtype=dtype) if weight is not None else dy
    dx = r * (g - xh * (g * xh).sum(axis=-1, keepdims=True) / C)
    dw = (dy * xh).reshape(-1, C).sum(axis=0) if weight is not None else None
    return dx, dw


def layernorm_fwd(x, weight=None, bias=None, eps=1e-5, dtype=np.float64):
    """y = (x - mean) / sqrt(var + eps) * weight + bias, biased var
    (src/scree/kernels/reference/varlen_layernorm.py:64-74)."""
    x = np.asarray(x, dtype=dtype)
    mean = x.mean(axis=-1, keepdims=True)
    var = x.var(axis=-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    if weight is not None:
        y = y * np.asarray(weight, dtype=dtype)
    if bias is not None:
        y = y + np.asarray(bias, dtype=dtype)
    return y


def layernorm_bwd(dy, x, weight=None, bias=None, eps=1e-5, dtype=np.float64):
    """(dx, dweight, dbias) of layernorm_fwd (None for absent parameters)."""
    x = np.asarray(x, dtype=dtype)
    dy = np.asarray(dy, dtype=dtype)
    C = x.shape[-1]
    mean = x.mean(axis=-1, keepdims=True)
    r = 1.0 / np.sqrt(x.var(axis=-1, keepdims=True) + eps)
    xh = (x - mean) * r
    g = dy * np.asarray(weight, dtype=dtype) if weight is not None else dy
    dx = r * (g - g.mean(axis=-1, keepdims=True) - xh * (g * xh).mean(axis=-1, keepdims=True))
    dw = (dy * xh).reshape(-1, C).sum(axis=0) if weight is not None else None
    db = dy.reshape(-1, C).sum(axis=0) if bias is not None else None
    return dx, dw, db


# --------------------------------------------------------------------------- softmax
def softmax_fwd(values, offsets, dtype=np.float64):
    """Per-sequence softmax along axis 0 (src/scree/kernels/reference/varlen_softmax.py:55-61)."""
    x = np.asarray(values, dtype=dtype)
    out = np.empty_like(x)
    for i in range(len(offsets) - 1):
        s0, e0 = int(offsets[i]), int(offsets[i + 1])
        if e0 == s0:
            continue
        row = x[s0:e0]
        ex = np.exp(row - row.max(axis=0, keepdims=True))
        out[s0:e0] = ex / ex.sum(axis=0, keepdims=True)
    return out


def softmax_bwd(dy, y, offsets, dtype=np.float64):
    """Gradient of softmax_fwd: dx = y * (dy - sum_rows(dy * y)) per sequence."""
    dy = np.asarray(dy, dtype=dtype)
    y = np.asarray(y, dtype=dtype)
    dx = np.empty_like(y)
    for i in range(len(offsets) - 1):
        s0, e0 = int(offsets[i]), int(offsets[i + 1])
        if e0 == s0:
            continue
        dx[s0:e0] = y[s0:e0] * (dy[s0:e0] - (dy[s0:e0] * y[s0:e0]).sum(axis=0, keepdims=True))
    return dx
