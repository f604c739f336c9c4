"""Shared helpers for the GPU parity tests (compare CUDA results with the oracle)."""

import numpy as np
import torch

import oracle

# Attention tolerance vs the fp64 oracle on the same 16-bit inputs: max abs
# 2e-3 for fp16, 1e-2 for bf16 (the north-star parity bar), plus the rounding
# of the result to its 16-bit storage type (half an ulp: 2^-12 relative for
# fp16, 2^-9 for bf16; a flat 1e-2 is finer than bf16 can represent once |x| >= 4).
ATTN_TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
ATTN_REL = {torch.float16: 2.0**-11, torch.bfloat16: 2.0**-8}


def excess(got, want, atol, rtol):
    """Largest |got - want| - (atol + rtol |want|); <= 0 means within bounds."""
    g = np.asarray(got, dtype=np.float64)
    w = np.asarray(want, dtype=np.float64)
    if g.size == 0:
        return -atol
    return float(np.max(np.abs(g - w) - (atol + rtol * np.abs(w))))


def to64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def offsets_np(lengths):
    o = np.zeros(len(lengths) + 1, dtype=np.int64)
    o[1:] = np.cumsum(lengths)
    return o


def attn_reference(q, k, v, do, lengths, causal, heads=None):
    """Oracle forward+backward on (a head subset of) the fp64 upcast of the GPU inputs."""
    sl = slice(None) if heads is None else heads
    qn, kn, vn, don = (to64(t[:, sl]) for t in (q, k, v, do))
    offs = offsets_np(lengths)
    out, lse = oracle.attention_fwd(qn, kn, vn, offs, causal=causal)
    dq, dk, dv = oracle.attention_bwd(don, qn, kn, vn, offs, causal=causal)
    return out, lse, dq, dk, dv


def max_err(a, b):
    return float(np.max(np.abs(np.asarray(a, dtype=np.float64) - np.asarray(b, dtype=np.float64)))) if np.size(a) else 0.0


def round_to(x, dtype):
    """Round float64 values to a torch 16-bit dtype and back."""
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).double().numpy()


def attn_bwd_emulated(do, q, k, v, lengths, causal, dtype):
    """Oracle backward evaluated with the 16-bit rounding points every tensor-core
    attention backward has (scree's Triton kernel included:
    triton/_backward.py:174, :181, :282): the forward output O is stored in
    `dtype` before Delta = rowsum(O * dO), and P and dS are rounded to `dtype`
    before their GEMMs.  Everything else is float64."""
    import math as _m

    qn, kn, vn, don = (to64(t) for t in (q, k, v, do))
    offs = offsets_np(lengths)
    out, _ = oracle.attention_fwd(qn, kn, vn, offs, causal=causal)
    out = round_to(out, dtype)
    scale = 1.0 / _m.sqrt(qn.shape[-1])
    dq, dk, dv = np.zeros_like(qn), np.zeros_like(kn), np.zeros_like(vn)
    for i in range(len(offs) - 1):
        s0, e0 = int(offs[i]), int(offs[i + 1])
        if e0 == s0:
            continue
        qh, kh, vh, doh, oh = (t[s0:e0].transpose(1, 0, 2) for t in (qn, kn, vn, don, out))
        sc = np.matmul(qh, kh.transpose(0, 2, 1)) * scale
        if causal:
            L = e0 - s0
            sc = np.where(np.triu(np.ones((L, L), dtype=bool), k=1), -np.inf, sc)
        m = sc.max(-1, keepdims=True)
        P = np.exp(sc - m)
        P /= P.sum(-1, keepdims=True)
        delta = (oh * doh).sum(-1, keepdims=True)
        Pr = round_to(P, dtype)
        dv[s0:e0] = np.matmul(Pr.transpose(0, 2, 1), doh).transpose(1, 0, 2)
        dP = np.matmul(doh, vh.transpose(0, 2, 1))
        dS = round_to(P * (dP - delta), dtype)
        dq[s0:e0] = (scale * np.matmul(dS, kh)).transpose(1, 0, 2)
        dk[s0:e0] = (scale * np.matmul(dS.transpose(0, 2, 1), qh)).transpose(1, 0, 2)
    return dq, dk, dv
