"""Whole-sequence sharding of a packed batch across ranks (one process per GPU).

Sequences are independent in every op of the varlen path (attention has no
cross-sequence term, norms are per token), so a batch splits across GPUs with
no reduction: each rank runs the kernels on its own sub-batch.  This module
holds the host side of that:

  * plan_shards   longest-processing-time-first assignment of sequences to
                  ranks by cost (L^2 for attention, L for norms / gathers);
  * broadcast_plan  rank 0's plan sent to every rank (torch.distributed, any
                  backend), with a check that every rank derived the same one;
  * LocalShard    a rank's sub-batch: its sequence indices, local offsets and
                  the global token rows they come from;
  * gather_to_rank0  per-rank outputs collected on rank 0 in global order
                  (point-to-point sends to rank 0 only);
  * plan_units    the same LPT over (sequence, head range) units: a sequence
                  whose attention cost exceeds a fraction of a rank's share is
                  split into equal head groups (each group's output rows are
                  disjoint, so this stays reduction-free) -- batches dominated
                  by one long sequence (cfg2, cfg5) balance this way.
Multi-GPU runs use NCCL over NVLink for these collectives; the CPU tests use gloo.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np

from .workloads import lpt_partition


def plan_shards(lengths: Sequence[int], world: int, cost: str = "attention") -> List[List[int]]:
    """Sequence indices per rank, balanced by L^2 ("attention") or L ("tokens")."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if cost == "attention":
        costs = [float(L) * float(L) for L in lengths]
    elif cost == "tokens":
        costs = [float(L) for L in lengths]
    else:
        raise ValueError(f"unknown cost model {cost!r}")
    return lpt_partition(costs, world)


def imbalance(lengths: Sequence[int], plan: List[List[int]], cost: str = "attention") -> float:
    """max rank cost / mean rank cost of a plan (1.0 = perfect)."""
    f = (lambda L: float(L) ** 2) if cost == "attention" else float
    loads = [sum(f(lengths[i]) for i in part) for part in plan]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0


def broadcast_plan(plan: List[List[int]], group=None) -> List[List[int]]:
    """Send rank 0's plan to every rank; if any rank had computed another, every
    rank raises the same RuntimeError (an all-reduce MAX of a mismatch flag, so
    no rank proceeds alone into the next collective)."""
    import torch
    import torch.distributed as dist

    obj = [plan]
    dist.broadcast_object_list(obj, src=0, group=group)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    flag = torch.tensor([0 if obj[0] == plan else 1], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    if int(flag.item()) != 0:
        raise RuntimeError("shard plan differs across ranks (inputs or seeds disagree)")
    return obj[0]


@dataclass(frozen=True)
class LocalShard:
    """One rank's part of a packed batch."""

    seqs: tuple          # global sequence indices, ascending
    lengths: tuple       # their lengths
    offsets: np.ndarray  # local (B_r + 1,) int64 offsets
    rows: np.ndarray     # global token row of each local row, (T_r,) int64

    @property
    def tokens(self) -> int:
        return int(self.offsets[-1])


def local_shard(global_offsets: Sequence[int], plan: List[List[int]], rank: int) -> LocalShard:
    go = np.asarray(global_offsets, dtype=np.int64)
    seqs = tuple(sorted(plan[rank]))
    lengths = tuple(int(go[i + 1] - go[i]) for i in seqs)
    offs = np.zeros(len(seqs) + 1, dtype=np.int64)
    offs[1:] = np.cumsum(lengths)
    rows = (
        np.concatenate([np.arange(go[i], go[i + 1], dtype=np.int64) for i in seqs])
        if seqs
        else np.zeros(0, dtype=np.int64)
    )
    return LocalShard(seqs, lengths, offs, rows)


def gather_to_rank0(local_values, shard: LocalShard, total_rows: int, group=None,
                    plan: List[List[int]] | None = None, global_offsets=None):
    """All ranks pass their (T_r, ...) values; rank 0 receives the (T, ...) tensor
    in global row order, other ranks receive None.

    Point-to-point: every rank r > 0 sends its rows to rank 0 (NCCL send/recv
    over NVLink on GPUs, gloo on CPU); no rank but 0 receives anything.  When
    ``plan`` and ``global_offsets`` are given, every rank derives all ranks'
    row lists from them and nothing but the values crosses the wire; otherwise
    the row counts and row indices are sent first."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = local_values.device
    feat = tuple(local_values.shape[1:])
    vals = local_values.contiguous()
    if plan is not None and global_offsets is not None:
        rows_of = [torch.as_tensor(local_shard(global_offsets, plan, r).rows, device=dev)
                   for r in range(world)]
        counts = [int(r_.shape[0]) for r_ in rows_of]
    else:
        n = torch.tensor([vals.shape[0]], dtype=torch.int64, device=dev)
        ns = [torch.zeros_like(n) for _ in range(world)] if rank == 0 else None
        dist.gather(n, ns, dst=0, group=group)
        counts = [int(c.item()) for c in ns] if rank == 0 else None
        rows_of = None
    g0 = dist.get_global_rank(group, 0) if group is not None else 0

    def gr(r):
        return dist.get_global_rank(group, r) if group is not None else r

    if rank != 0:
        ops = []
        if vals.shape[0]:
            ops.append(dist.P2POp(dist.isend, vals, g0, group))
        if rows_of is None:
            my_rows = torch.as_tensor(shard.rows, dtype=torch.int64, device=dev)
            if my_rows.shape[0]:
                ops.append(dist.P2POp(dist.isend, my_rows, g0, group))
        for w in dist.batch_isend_irecv(ops) if ops else []:
            w.wait()
        return None
    bufs, rbufs, ops = {}, {}, []
    for r in range(1, world):
        if counts[r] == 0:
            continue
        bufs[r] = torch.empty((counts[r], *feat), dtype=vals.dtype, device=dev)
        ops.append(dist.P2POp(dist.irecv, bufs[r], gr(r), group))
        if rows_of is None:
            rbufs[r] = torch.empty((counts[r],), dtype=torch.int64, device=dev)
            ops.append(dist.P2POp(dist.irecv, rbufs[r], gr(r), group))
    for w in dist.batch_isend_irecv(ops) if ops else []:
        w.wait()
    out = torch.empty((total_rows, *feat), dtype=vals.dtype, device=dev)
    mine = rows_of[0] if rows_of is not None else torch.as_tensor(shard.rows, dtype=torch.int64, device=dev)
    if mine.shape[0]:
        out.index_copy_(0, mine, vals)
    for r, b in bufs.items():
        idx = rows_of[r] if rows_of is not None else rbufs[r]
        out.index_copy_(0, idx, b)
    return out


class GatherPlan:
    """Precomputed exchange of per-rank outputs to rank 0 for a whole-sequence
    plan: every sequence's rows travel as one contiguous message, straight into
    its slice of rank 0's global-order output (no staging buffer, no scatter of
    received rows), and all tensors of a step go in one batch of NCCL
    send/recv operations.  Rank 0's own rows are placed with one index copy."""

    def __init__(self, plan: List[List[int]], global_offsets, rank: int, device, group=None):
        import torch

        self.group = group
        self.rank = rank
        self.go = np.asarray(global_offsets, dtype=np.int64)
        self.total = int(self.go[-1])
        self.world = len(plan)
        # (peer rank, local row range, global row range) per sequence
        self.msgs = []
        for r, part in enumerate(plan):
            lo = 0
            for i in sorted(part):
                n = int(self.go[i + 1] - self.go[i])
                if n and r != 0:
                    self.msgs.append((r, lo, lo + n, int(self.go[i]), int(self.go[i + 1])))
                lo += n
        self.own_rows = torch.as_tensor(local_shard(self.go, plan, 0).rows, device=device)

    def _peer(self, r):
        import torch.distributed as dist

        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def run(self, tensors, defer: bool = False):
        """All ranks pass their local (T_r, ...) tensors; rank 0 gets the global
        (T, ...) tensors back, other ranks None.  With ``defer`` the pending
        requests are returned too, ``(outs, reqs)``: the transfer then overlaps
        whatever the caller enqueues next, and the caller waits on ``reqs``
        before it uses the outputs or frees the inputs."""
        import torch
        import torch.distributed as dist

        ops, outs = [], None
        if self.rank == 0:
            outs = [torch.empty((self.total, *t.shape[1:]), dtype=t.dtype, device=t.device) for t in tensors]
            for r, l0, l1, g0, g1 in self.msgs:
                for o in outs:
                    ops.append(dist.P2POp(dist.irecv, o[g0:g1], self._peer(r), self.group))
        else:
            srcs = [t.contiguous() for t in tensors]
            for r, l0, l1, g0, g1 in self.msgs:
                if r == self.rank:
                    for t in srcs:
                        ops.append(dist.P2POp(dist.isend, t[l0:l1], self._peer(0), self.group))
        reqs = dist.batch_isend_irecv(ops) if ops else []
        if self.rank == 0 and self.own_rows.numel():
            for o, t in zip(outs, tensors):
                o.index_copy_(0, self.own_rows, t)
        if defer:
            return outs, reqs
        for q in reqs:
            q.wait()
        return outs


@dataclass(frozen=True)
class Unit:
    """Attention work on heads [h0, h1) of one sequence."""

    seq: int
    h0: int
    h1: int

    @property
    def heads(self) -> int:
        return self.h1 - self.h0


def plan_units(lengths: Sequence[int], world: int, heads: int, split_frac: float = 0.25,
               max_groups: int = 2) -> List[List[Unit]]:
    """Units per rank.  A sequence of cost L^2 * heads above split_frac times the
    mean rank cost is cut into g equal head groups, g the smallest power of two
    (at most max_groups, dividing heads) that brings each group under that
    limit; units are then placed longest-first (LPT) on L^2 * (h1 - h0).
    max_groups defaults to 2: every head group feeds a separate attention call
    whose grid is tiles x heads, and measured on 4 B200s at cfg5, units of 1-2
    heads left so few CTAs per call that the step took twice as long as with
    whole sequences."""
    if world < 1 or heads < 1:
        raise ValueError("world and heads must be >= 1")
    total = sum(float(L) * float(L) * heads for L in lengths)
    limit = split_frac * total / world
    units: List[Unit] = []
    for i, L in enumerate(lengths):
        cost = float(L) * float(L) * heads
        g = 1
        while g < max_groups and heads % (2 * g) == 0 and cost / g > limit:
            g *= 2
        hs = heads // g
        units.extend(Unit(i, k * hs, (k + 1) * hs) for k in range(g))
    costs = [float(lengths[u.seq]) ** 2 * u.heads for u in units]
    return [[units[j] for j in part] for part in lpt_partition(costs, world)]


def units_imbalance(lengths: Sequence[int], plan: List[List[Unit]]) -> float:
    """max rank cost / mean rank cost of a unit plan (1.0 = perfect)."""
    loads = [sum(float(lengths[u.seq]) ** 2 * u.heads for u in part) for part in plan]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0


def units_by_heads(plan_rank: List[Unit]):
    """A rank's units grouped by head count: {heads: [Unit, ...]} in sequence
    order; each group runs as one attention call over its sequences."""
    out = {}
    for u in sorted(plan_rank, key=lambda u: (u.seq, u.h0)):
        out.setdefault(u.heads, []).append(u)
    return out
