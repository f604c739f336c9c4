"""Seeded synthetic workloads for the five benchmark configurations.

Sequence lengths follow the reference's sampler (benchmarks/bench_throughput.py:31-34:
``rng.lognormal(log(mean), sigma)``) with numpy's ``default_rng(seed)``; values
are drawn in fp32 from ``torch.Generator`` seeded with the same seed and then
cast.  There is no dataset: every config is synthetic.

  cfg1  16 seqs, mean 110,  sigma 0.6, max(1, round(.)),  H4  D32  fp32
  cfg2  16 seqs, mean 700,  sigma 0.6, rescaled to sum exactly 12160, H16 D64 fp16
  cfg3  64 seqs, mean 256,  sigma 0.6, hidden 4096 bf16 (norms, pack/unpack)
  cfg4  64 seqs, mean 2048, sigma 0.6, clipped [16, 16384], H32 D128 bf16
  cfg5  32 seqs, mean 1024, sigma 1.2, clipped [1, 32768], first 4 forced to 1, H16 D128 bf16
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List

import numpy as np


@dataclass(frozen=True)
class AttnConfig:
    name: str
    lengths: tuple
    heads: int
    head_dim: int
    dtype: str
    causal: bool

    @property
    def total(self) -> int:
        return int(sum(self.lengths))


def _lognormal(n, mean, sigma, seed):
    rng = np.random.default_rng(seed)
    return rng.lognormal(mean=math.log(mean), sigma=sigma, size=n)


def cfg1_lengths(seed=0) -> List[int]:
    return [max(1, int(round(x))) for x in _lognormal(16, 110, 0.6, seed)]


def cfg2_lengths(seed=0, total=12160) -> List[int]:
    raw = _lognormal(16, 700, 0.6, seed)
    scaled = raw * (total / raw.sum())
    base = np.maximum(1, np.floor(scaled)).astype(np.int64)
    rem = int(total - base.sum())
    order = np.argsort(-(scaled - np.floor(scaled)))
    for i in range(abs(rem)):
        base[order[i % len(base)]] += 1 if rem > 0 else -1
    assert int(base.sum()) == total
    return [int(x) for x in base]


def cfg3_lengths(seed=0) -> List[int]:
    return [max(1, int(round(x))) for x in _lognormal(64, 256, 0.6, seed)]


def cfg4_lengths(seed=0) -> List[int]:
    return [int(np.clip(round(x), 16, 16384)) for x in _lognormal(64, 2048, 0.6, seed)]


def cfg5_lengths(seed=0) -> List[int]:
    ls = [int(np.clip(round(x), 1, 32768)) for x in _lognormal(32, 1024, 1.2, seed)]
    ls[:4] = [1, 1, 1, 1]
    return ls


def attn_config(name: str, seed: int = 0, causal: bool = True) -> AttnConfig:
    if name == "cfg1":
        return AttnConfig("cfg1", tuple(cfg1_lengths(seed)), 4, 32, "float32", causal)
    if name == "cfg2":
        return AttnConfig("cfg2", tuple(cfg2_lengths(seed)), 16, 64, "float16", causal)
    if name == "cfg4":
        return AttnConfig("cfg4", tuple(cfg4_lengths(seed)), 32, 128, "bfloat16", causal)
    if name == "cfg5":
        return AttnConfig("cfg5", tuple(cfg5_lengths(seed)), 16, 128, "bfloat16", causal)
    raise KeyError(name)


def causal_pairs(lengths) -> int:
    return int(sum(L * (L + 1) // 2 for L in lengths))


def attn_flops(lengths, heads, head_dim, causal=True, fwd=True, bwd=True) -> float:
    """Algorithmic FLOPs: 4*H*D*pairs forward, 10*H*D*pairs backward (5 GEMMs),
    pairs = L(L+1)/2 causal or L^2 non-causal per sequence."""
    pairs = causal_pairs(lengths) if causal else int(sum(L * L for L in lengths))
    f = 0.0
    if fwd:
        f += 4.0 * heads * head_dim * pairs
    if bwd:
        f += 10.0 * heads * head_dim * pairs
    return f


def offsets_of(lengths) -> np.ndarray:
    off = np.zeros(len(lengths) + 1, dtype=np.int64)
    off[1:] = np.cumsum(lengths)
    return off


def make_qkv(lengths, heads, head_dim, dtype, device, seed=0, with_do=True):
    """q, k, v (and dO) ~ N(0,1) drawn in fp32 from torch.Generator(seed), cast."""
    import torch

    T = int(sum(lengths))
    g = torch.Generator(device="cpu").manual_seed(seed)
    dt = getattr(torch, dtype) if isinstance(dtype, str) else dtype
    out = []
    for _ in range(4 if with_do else 3):
        t = torch.randn((T, heads, head_dim), generator=g, dtype=torch.float32)
        out.append(t.to(dt).to(device))
    return out


def lpt_partition(costs, n_parts):
    """Longest-processing-time-first assignment of items to n_parts bins;
    returns a list of index lists (each sorted)."""
    order = sorted(range(len(costs)), key=lambda i: -costs[i])
    loads = [0.0] * n_parts
    parts = [[] for _ in range(n_parts)]
    for i in order:
        j = min(range(n_parts), key=lambda p: loads[p])
        parts[j].append(i)
        loads[j] += costs[i]
    return [sorted(p) for p in parts]
