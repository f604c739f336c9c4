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
