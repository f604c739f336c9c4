"""Attention parity cases and their error measurement, shared by the GPU tests
(tests/test_gpu_attention.py) and the error-table generator
(tests/attn_error_table.py).

Bar: max-abs error against the fp64 oracle on the same
16-bit inputs of at most 2e-3 (fp16) / 1e-2 (bf16) for the attention output and
its gradients, plus the rounding of a result to its 16-bit storage type (one
ulp of headroom relative: 2^-11 fp16, 2^-8 bf16 -- a flat 1e-2 is finer than
bf16 can hold once |x| >= 4).  LSE (fp32): 1e-3 absolute.

A gradient that misses that bound passes only when the bound is shown to be
out of reach for any tensor-core backward on the case: the fp64 oracle
evaluated with the 16-bit rounding points of such a backward (O stored in 16
bits, P and dS rounded to 16 bits before their GEMMs -- scree's own Triton
backward has them too, triton/_backward.py:174, :181, :282) must itself miss
the bound, and the kernel's error must be at most twice that emulation's.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

import oracle
from gpu_helpers import ATTN_REL, ATTN_TOL, attn_bwd_emulated, attn_reference, excess, max_err, to64

EDGE_LENGTHS = [
    [1],
    [1, 1, 1],
    [2, 3],
    [127, 128, 129],
    [255, 1, 257],
    [5, 0, 9, 300],
    [64, 17, 200, 33],
]

NAMES = ("out", "lse", "dq", "dk", "dv")


@dataclass
class Stat:
    name: str
    max_abs: float
    flat: float          # the flat bound (1e-2 bf16 / 2e-3 fp16 / 1e-3 LSE)
    flat_ok: bool        # max_abs <= flat
    bound_excess: float  # max(|err| - (flat + rel |ref|)); <= 0 within the bound
    emul: float | None = None          # max-abs error of the 16-bit-operand emulation
    emul_excess: float | None = None   # its excess over the same bound

    @property
    def bound_ok(self) -> bool:
        return self.bound_excess <= 0

    @property
    def verdict(self) -> str:
        if self.bound_ok:
            return "within bound"
        if self.emul is not None and self.emul_excess is not None and self.emul_excess > 0 \
                and self.max_abs <= 2 * self.emul:
            return "bound unreachable: emulation misses it, kernel <= 2x emulation"
        return "FAIL"


@dataclass
class CaseResult:
    case: str
    dtype: str
    stats: list = field(default_factory=list)

    def failures(self):
        return [s for s in self.stats if s.verdict == "FAIL"]


def _stats_for(name_prefix, outs, ref, ins, lengths, causal, dtype, check_bwd=True):
    tol, rel = ATTN_TOL[dtype], ATTN_REL[dtype]
    res = []
    emul = None
    for name, got, want in zip(NAMES, outs, ref):
        if got is None or (not check_bwd and name in ("dq", "dk", "dv")):
            continue
        g = to64(got)
        if name == "lse":
            st = Stat(name, max_err(g, want), 1e-3, max_err(g, want) <= 1e-3, excess(g, want, 1e-3, 0.0))
        else:
            e = max_err(g, want)
            st = Stat(name, e, tol, e <= tol, excess(g, want, tol, rel))
        if name in ("dq", "dk", "dv") and not st.bound_ok:
            if emul is None:
                emul = dict(zip(("dq", "dk", "dv"), attn_bwd_emulated(*ins, lengths, causal, dtype)))
            st.emul = max_err(emul[name], want)
            st.emul_excess = excess(emul[name], want, tol, rel)
        res.append(st)
    return res


def run_kernels(q, k, v, do, cu, causal, with_bwd=True):
    from scree_b200.kernels.native import varlen_attention_triton, varlen_attention_triton_backward

    out, lse = varlen_attention_triton(q, k, v, cu, causal=causal, return_lse=True)
    if not with_bwd:
        torch.cuda.synchronize()
        return out, lse, None, None, None
    dq, dk, dv = varlen_attention_triton_backward(do, q, k, v, out, lse, cu, causal=causal)
    torch.cuda.synchronize()
    return out, lse, dq, dk, dv


def measure(lengths, H, D, dtype, causal, device, heads=None, seed=0, offs_dtype=torch.int32):
    """Run the kernels on the whole batch; compare (a head subset of) every output."""
    from scree_b200 import workloads

    q, k, v, do = workloads.make_qkv(lengths, H, D, dtype, device, seed=seed)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=offs_dtype, device=device)
    outs = run_kernels(q, k, v, do, cu, causal)
    sl = slice(None) if heads is None else heads
    ins = [t[:, sl] for t in (q, k, v, do)]
    ref = attn_reference(*ins, lengths, causal)
    return _stats_for("", [o[:, sl] for o in outs], ref, [ins[3], ins[0], ins[1], ins[2]], lengths, causal, dtype)


def measure_sampled(lengths, H, D, dtype, causal, device, seqs, heads, seed=0, with_bwd=True):
    """Run the kernels on the whole batch; compare the listed (sequence, head)
    pairs one at a time (full-size configs).  Returns {(seq, head): [Stat]} and
    the raw outputs."""
    from scree_b200 import workloads

    q, k, v, do = workloads.make_qkv(lengths, H, D, dtype, device, seed=seed)
    offs = np.concatenate([[0], np.cumsum(lengths)])
    cu = torch.tensor(offs, dtype=torch.int32, device=device)
    outs = run_kernels(q, k, v, do, cu, causal, with_bwd)
    for t in outs:
        if t is not None:
            assert torch.isfinite(t).all()
    first = torch.tensor(offs[:-1], device=device, dtype=torch.long)
    # Causal known answer: a sequence's first output row is its first V row.
    if causal:
        assert torch.equal(outs[0][first], v[first])
    res = {}
    for b in seqs:
        s, e = int(offs[b]), int(offs[b + 1])
        for h in heads:
            sub = [t[s:e, h : h + 1] for t in (q, k, v, do)]
            got = [None if t is None else t[s:e, h : h + 1] for t in outs]
            qn, kn, vn = (to64(t) for t in sub[:3])
            if with_bwd:
                ref = attn_reference(*sub, [e - s], causal)
            else:
                ro, rl = oracle.attention_fwd(qn, kn, vn, [0, e - s], causal=causal)
                ref = (ro, rl, None, None, None)
            res[(b, h)] = _stats_for("", got, ref, [sub[3], sub[0], sub[1], sub[2]], [e - s], causal,
                                     dtype, check_bwd=with_bwd)
    return res


def sample_seqs(lengths, n):
    """n sequence indices spread over the length distribution (shortest and longest included)."""
    order = np.argsort(lengths, kind="stable")
    if n >= len(order):
        return [int(i) for i in order]
    picks = np.linspace(0, len(order) - 1, n).round().astype(int)
    return sorted({int(order[p]) for p in picks})
