"""Shared helpers for the GPU parity tests (compare CUDA results with the oracle)."""

import numpy as np
import torch

import oracle

# Attention tolerance (max abs vs the fp64 oracle on the same 16-bit inputs):
# 2e-3 for fp16, 1e-2 for bf16, as the north-star parity bar states.
ATTN_TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


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
