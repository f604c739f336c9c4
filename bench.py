#!/usr/bin/env python
"""Varlen attention fwd+bwd throughput of scree_b200 on B200 (one JSON line).

    python bench.py [--gpus N --steps K --warmup W] [--impl native|reference]

Workload (default): cfg4 — 64 sequences, lengths lognormal(ln 2048, 0.6) clipped
to [16, 16384] at seed 0 (T = 158,330 tokens), q/k/v/dO ~ N(0,1) bf16 of shape
(T, 32 heads, 128), causal.  A step is one forward + backward through the
drop-in autograd entry point (varlen_attention_triton_autograd -> out.backward).
At cfg4 every q/k/v/dO tensor is 1.3 GB, far larger than the 126 MB L2, so no
flush is needed between steps; when a rank's tensors are under 256 MB (cfg2,
cfg5, cfg4 split 8 ways) a 256 MB buffer is written before every timed step,
outside that step's CUDA events.

Multi-GPU (torchrun, one process per GPU): the fixed batch is split by whole
sequences, longest-processing-time-first on L^2, identically on every rank (the
plan is broadcast from rank 0 over NCCL as a consistency check).  There is no
collective on the data path; the step time is the max over ranks (CUDA events,
all_reduce MAX) and ``value`` = all tokens / that time ("strong" scaling: total
work fixed).

--impl reference times the reference algorithm on the host CPU instead: the
numpy oracle (a restatement of scree.kernels.reference; the reference itself is
pure Python and is not installed on the GPU box), fp32, all host cores, on a
bounded sample of cfg4's sequences, extrapolated to the whole workload by
algorithmic FLOPs.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "varlen-attn fwd+bwd tokens/s & TFLOP/s vs TC peak at 1/2/4/8 B200"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 * 1024 * 1024  # 2x the 126 MB L2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


# ----------------------------------------------------------------------------- clocks
_REASONS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x10: "sync_boost",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


class ClockSampler:
    """Samples SM clock and clock-event reasons every 200 ms through NVML (read only)."""

    def __init__(self, device_index: int):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            handle = None
            try:
                import torch

                props = torch.cuda.get_device_properties(device_index)
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._h = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            self._stop.wait(0.2)

    def start(self):
        if self.ok:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= int(r)
        reasons = [name for b, name in _REASONS.items() if bits & b and name != "gpu_idle"]
        return {
            "sm_mhz": float(statistics.median(mhz)),
            "sm_max_mhz": self.max_mhz,
            "reasons": reasons,
            "samples": len(mhz),
        }


# ----------------------------------------------------------------------------- CPU arm
def cpu_reference_rate(lengths, H, D, causal, budget_s=12.0, repeats=2, log=None):
    """Time the oracle (numpy fp32, all host cores) forward+backward on a bounded
    sample of the workload's sequences and extrapolate to the whole workload by
    algorithmic FLOPs.  Returns (tokens/s, cores, sample description)."""
    import oracle
    from scree_b200 import workloads

    cores = len(os.sched_getaffinity(0))
    T_total = sum(lengths)
    F_total = workloads.attn_flops(lengths, H, D, causal)
    # Sample: the median-length sequence, all heads (cost per token of the batch
    # is dominated by pair count, which the FLOP scaling accounts for).
    order = np.argsort(lengths)
    L = int(lengths[int(order[len(order) // 2])])
    rng = np.random.default_rng(0)
    q, k, v, do = (rng.standard_normal((L, H, D)).astype(np.float32) for _ in range(4))
    offs = [0, L]

    def run():
        oracle.attention_fwd(q, k, v, offs, causal=causal, dtype=np.float32)
        oracle.attention_bwd(do, q, k, v, offs, causal=causal, dtype=np.float32)

    run()  # warm-up
    times = []
    t_start = time.perf_counter()
    for _ in range(repeats):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    t = statistics.median(times)
    F_sample = workloads.attn_flops([L], H, D, causal)
    rate = T_total / (t * F_total / F_sample)
    sample = (f"one sequence of L={L} (cfg4 median) x {H} heads x D={D}, fp32 numpy oracle "
              f"fwd+bwd, median of {len(times)} after 1 warm-up = {t:.3f} s; extrapolated to "
              f"all {len(lengths)} sequences by algorithmic FLOPs ({F_total / F_sample:.1f}x)")
    return rate, cores, sample


def run_reference_arm(args, lengths, H, D, causal):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    from scree_b200 import workloads

    cores = len(os.sched_getaffinity(0))
    order = np.argsort(lengths)
    L = int(lengths[int(order[len(order) // 2])])
    rng = np.random.default_rng(0)
    q, k, v, do = (rng.standard_normal((L, H, D)).astype(np.float32) for _ in range(4))
    offs = [0, L]

    def step():
        oracle.attention_fwd(q, k, v, offs, causal=causal, dtype=np.float32)
        oracle.attention_bwd(do, q, k, v, offs, causal=causal, dtype=np.float32)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    T_total = sum(lengths)
    F_total = workloads.attn_flops(lengths, H, D, causal)
    F_sample = workloads.attn_flops([L], H, D, causal)
    step_full = dt * F_total / F_sample
    value = T_total / step_full
    sample = (f"each step: one sequence of L={L} (cfg4 median) x {H} heads x D={D}, numpy oracle "
              f"(restatement of scree.kernels.reference) fp32 fwd+bwd on {cores} host threads, "
              f"extrapolated to the whole workload by algorithmic FLOPs ({F_total / F_sample:.1f}x)")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_full * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(args, lengths, H, D, causal, world),
        "tflops": F_total / step_full / 1e12,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


_LEN_DESC = {
    "cfg2": "lognormal(ln 700, 0.6) rescaled to 12160 tokens",
    "cfg4": "lognormal(ln 2048, 0.6) clip [16,16384]",
    "cfg5": "lognormal(ln 1024, 1.2) clip [1,32768], 4 forced length-1",
}


def workload_config(args, lengths, H, D, causal, world):
    return {
        "workload": f"{args.config}: {len(lengths)} seqs {_LEN_DESC[args.config]} seed 0, "
        f"T={sum(lengths)}, H={H}, D={D}, {getattr(args, 'dtype_name', 'bfloat16')}, {'causal' if causal else 'non-causal'} fwd+bwd",
        "global_batch": int(sum(lengths)),
        "seqs": len(lengths),
        "max_seqlen": int(max(lengths)),
        "heads": H,
        "head_dim": D,
        "causal": causal,
        "parallelism": (f"{'head-group' if getattr(args, 'shard', 'seqs') == 'heads' else 'seq'}-shard{world}"
                        if world > 1 else "single"),
        "l2": getattr(args, "l2_note", "inputs larger than L2"),
    }


# ----------------------------------------------------------------------------- norms suite
def run_norm_suite(args):
    """cfg3: 64 sequences, lengths lognormal(ln 256, 0.6) (T = 19,794), hidden 4096
    bf16.  Each op is timed per launch with CUDA events; a 256 MB buffer is
    written between launches to flush the 126 MB L2.  Bandwidth = algorithmic
    bytes (reads + writes the op must do) / time, against MEASURED_PEAKS hbm_gbs."""
    import torch

    import scree_b200 as scree
    from scree_b200 import _lib, workloads
    from scree_b200.kernels import native

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lengths = workloads.cfg3_lengths()
    T, C, b = sum(lengths), 4096, 2
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((T, C), device=dev, generator=g).to(torch.bfloat16)
    dy = torch.randn((T, C), device=dev, generator=g).to(torch.bfloat16)
    w = (1 + 0.02 * torch.randn(C, device=dev, generator=g))
    bias = 0.02 * torch.randn(C, device=dev, generator=g)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
    arr = scree.from_cu_seqlens(x, offs)
    rows = scree.unpack(arr)
    Lmax = max(lengths)
    padded, mask = scree.to_padded(arr)
    _, rstd = native._rmsnorm_fwd(x, w, 1e-5, True)
    _, mean, rstd_l = native._layernorm_fwd(x, w, bias, 1e-5, True)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    sm_y = native.varlen_softmax_packed(x, offs)
    sm_dx = torch.empty_like(x)
    B = len(lengths)
    ops = {
        "rmsnorm_fwd": (lambda: native.varlen_rmsnorm_triton(x, w, 1e-5), 2 * T * C * b + 4 * C),
        "rmsnorm_bwd": (lambda: native.varlen_rmsnorm_backward(dy, x, w, rstd), 3 * T * C * b + 4 * T + 4 * C),
        "layernorm_fwd": (lambda: native.varlen_layernorm_triton(x, w, bias, 1e-5), 2 * T * C * b + 8 * C),
        "layernorm_bwd": (lambda: native.varlen_layernorm_backward(dy, x, w, bias, mean, rstd_l), 3 * T * C * b + 8 * T + 8 * C),
        "pack": (lambda: scree.pack(rows), 2 * T * C * b + 4 * (B + 1)),
        "to_padded": (lambda: scree.to_padded(arr), T * C * b + B * Lmax * C * b + B * Lmax),
        "from_padded": (lambda: scree.from_padded(padded, mask), B * Lmax + 2 * T * C * b),
        "softmax_fwd": (lambda: native.varlen_softmax_packed(x, offs), 2 * T * C * b),
        "softmax_bwd": (lambda: native._softmax_call(_lib.load().scree_softmax_bwd, "sm bwd", offs, sm_dx, dy, sm_y), 3 * T * C * b),
    }
    peaks, kind = load_peaks()
    hbm = float(peaks["hbm_gbs"])
    res = {}
    for name, (fn, nbytes) in ops.items():
        for _ in range(max(3, args.warmup)):
            fn()
        # Kernel-only time from the library's CUDA-event hooks around each
        # launch; the 256 MB flush is written before every launch.
        # (the softmax kernels report under the norm fwd / bwd event kinds)
        kind_ = _lib.PROF_NORM_FWD if name.endswith("_fwd") else (_lib.PROF_NORM_BWD if name.endswith("_bwd") else _lib.PROF_GATHER)
        times = []
        _lib.profile_read(kind_)
        _lib.profile_enable(True)
        for _ in range(args.steps):
            flush.fill_(1)
            fn()
            torch.cuda.synchronize()
            tms, nl = _lib.profile_read(kind_)
            times.append(tms / max(nl, 1) * max(nl, 1))  # all launches of one call
        _lib.profile_enable(False)
        ms = statistics.median(times)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"ms": ms, "algorithmic_bytes": int(nbytes), "gb_s": gbs, "frac": gbs / hbm}
    assert _lib.device_status() == 0
    cpu = None
    if not args.no_cpu_baseline:
        import oracle

        xn = x.float().cpu().numpy()
        wn = w.cpu().numpy()
        oracle.rmsnorm_fwd(xn, wn, 1e-5, dtype=np.float32)
        t0 = time.perf_counter()
        oracle.rmsnorm_fwd(xn, wn, 1e-5, dtype=np.float32)
        t_cpu = time.perf_counter() - t0
        cpu = {"value": 2 * T * C * b / t_cpu / 1e9, "unit": "GB/s", "cores": len(os.sched_getaffinity(0)),
               "kind": "port", "sample": f"rmsnorm_fwd on the full cfg3 batch (fp32 numpy oracle), {t_cpu:.3f} s"}
    line = {
        "metric": "varlen norms / softmax / gathers HBM GB/s (cfg3)",
        "value": res["rmsnorm_fwd"]["gb_s"],
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": max(3, args.warmup),
        "higher_is_better": True,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"cfg3: 64 seqs lognormal(ln 256, 0.6) seed 0, T={T}, hidden {C} bf16",
                   "l2": "256 MB buffer written before every timed call", "timing": "kernel time from CUDA events around each launch inside libscree_b200 (all launches of the call summed)"},
        "ops": res,
        "hbm_peak_gbs": hbm,
        "peak_source": kind,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--config", default="cfg4", choices=["cfg4", "cfg2", "cfg5"])
    ap.add_argument("--e2e-steps", type=int, default=6)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--non-causal", action="store_true")
    ap.add_argument("--shard", choices=["seqs", "heads"], default="seqs",
                    help="multi-GPU split: whole sequences (default) or sequences split by head groups")
    ap.add_argument("--suite", choices=["attention", "norms"], default="attention",
                    help="norms: cfg3 RMSNorm/LayerNorm fwd+bwd and pack/unpack/to_padded/from_padded")
    ap.add_argument("--max-seqs", type=int, default=0, help="keep only the first N sequences (small profiling case)")
    args = ap.parse_args()

    from scree_b200 import workloads

    if args.suite == "norms":
        run_norm_suite(args)
        return
    cfg = workloads.attn_config(args.config)
    lengths = list(cfg.lengths)
    if args.max_seqs:
        lengths = lengths[: args.max_seqs]
    H, D, causal = cfg.heads, cfg.head_dim, cfg.causal and not args.non_causal
    args.dtype_name = "float16" if cfg.dtype == "float16" else "bfloat16"

    if args.impl == "reference":
        run_reference_arm(args, lengths, H, D, causal)
        return

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    from scree_b200 import _lib
    from scree_b200.kernels.native import varlen_attention_triton_autograd

    # Shard plan, broadcast from rank 0: whole sequences by LPT on L^2, or
    # (--shard heads) (sequence, head group) units; a rank runs one attention
    # call per head count among its units.
    from scree_b200 import shard

    if args.shard == "heads":
        plan = shard.plan_units(lengths, world, H)
        if world > 1:
            plan = shard.broadcast_plan(plan)
        groups = [(hs, [lengths[u.seq] for u in us])
                  for hs, us in sorted(shard.units_by_heads(plan[rank]).items(), reverse=True)]
        args.no_e2e = True  # the end-to-end path is measured on whole sequences
    else:
        plan = shard.plan_shards(lengths, world, cost="attention")
        if world > 1:
            plan = shard.broadcast_plan(plan)
        groups = [(H, [lengths[i] for i in sorted(plan[rank])])]
    # Tokens this rank covers: a sequence split over head groups counts its
    # length times the fraction of heads each unit holds.
    T = sum(sum(ls) * hs / H for hs, ls in groups)
    dt = getattr(torch, args.dtype_name)
    g = torch.Generator(device=dev).manual_seed(1234 + 17 * rank)

    calls = []  # (q, k, v, dO, cu) per head-count group
    for hs, ls in groups:
        Tg = sum(ls)

        def rnd():
            return torch.randn((Tg, hs, D), device=dev, dtype=torch.float32, generator=g).to(dt)

        qg, kg, vg, dog = rnd(), rnd(), rnd(), rnd()
        for t in (qg, kg, vg):
            t.requires_grad_(True)
        cug = torch.tensor(np.concatenate([[0], np.cumsum(ls)]), dtype=torch.int32, device=dev)
        calls.append((qg, kg, vg, dog, cug))
    q, k, v, do, cu = calls[0]  # whole-sequence mode: the only group

    def step():
        for qg, kg, vg, dog, cug in calls:
            for t in (qg, kg, vg):
                t.grad = None
            out = varlen_attention_triton_autograd(qg, kg, vg, cug, causal=causal)
            out.backward(dog)

    tensor_bytes = sum(qg.numel() for qg, *_ in calls) * q.element_size()
    flush = None
    if tensor_bytes < L2_FLUSH_BYTES:
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    args.l2_note = (f"inputs larger than L2 (each of q/k/v/dO {tensor_bytes / 1e6:.0f} MB per rank)"
                    if flush is None else
                    f"q/k/v/dO {tensor_bytes / 1e6:.0f} MB each per rank: 256 MB buffer written before every timed step, outside its events")

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    _lib.profile_read(_lib.PROF_ATTN_FWD)
    _lib.profile_read(_lib.PROF_ATTN_BWD)
    _lib.profile_enable(True)
    n0 = _lib.launch_count()
    if flush is None:
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(args.steps):
            step()
        ev1.record()
        torch.cuda.synchronize()
        elapsed_ms = ev0.elapsed_time(ev1)
    else:
        # Inputs fit in L2: a 256 MB buffer is written before every step, outside
        # that step's event pair; the steps' own device times are summed.
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for a, b in evs:
            flush.fill_(1)
            a.record()
            step()
            b.record()
        torch.cuda.synchronize()
        elapsed_ms = sum(a.elapsed_time(b) for a, b in evs)
    launches = _lib.launch_count() - n0
    _lib.profile_enable(False)
    fwd_ms, nf = _lib.profile_read(_lib.PROF_ATTN_FWD)
    bwd_ms, nb = _lib.profile_read(_lib.PROF_ATTN_BWD)
    if world > 1:
        dist.barrier()
    sampler.stop()
    assert _lib.device_status() == 0, "kernel reported an error (device status word)"

    flops_mine = sum(workloads.attn_flops(ls, hs, D, causal) for hs, ls in groups)
    flops_fwd_mine = sum(workloads.attn_flops(ls, hs, D, causal, fwd=True, bwd=False) for hs, ls in groups)
    flops_bwd_mine = sum(workloads.attn_flops(ls, hs, D, causal, fwd=False, bwd=True) for hs, ls in groups)
    stats = torch.tensor([elapsed_ms, float(T), flops_mine, float(launches)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = stats.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        max_ms, total_T, total_flops, total_launch = float(mx[0]), float(sm[1]), float(sm[2]), float(sm[3])
    else:
        max_ms, total_T, total_flops, total_launch = elapsed_ms, float(T), flops_mine, float(launches)
    ms_step = max_ms / args.steps
    value = total_T / (ms_step / 1e3)
    tflops = total_flops / (ms_step / 1e3) / 1e12

    peaks, peak_kind = load_peaks()
    peak_tf = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    bwd_avg_ms = bwd_ms / max(nb, 1)
    fwd_avg_ms = fwd_ms / max(nf, 1)
    # This rank's FLOPs per step over its kernel time per step (one launch per
    # step and kind, or one per head-count group with --shard heads).
    ach_bwd = flops_bwd_mine / (bwd_ms / args.steps / 1e3) / 1e12
    ach_fwd = flops_fwd_mine / (fwd_ms / args.steps / 1e3) / 1e12
    traffic = None
    tp = ROOT / "profiles" / "attn_bwd_cfg4_traffic.json"
    if tp.exists():
        try:
            traffic = json.loads(tp.read_text()).get("bytes_per_launch")
        except Exception:
            traffic = None

    # ------------------------------------------------------------ end to end
    e2e = None
    if not args.no_e2e:
        hq, hk, hv, hdo = (t.detach().cpu().pin_memory() for t in (q, k, v, do))
        ho = torch.empty_like(hq).pin_memory()
        hdq, hdk, hdv = (torch.empty_like(hq).pin_memory() for _ in range(3))
        # Pipelined steps: step i's host->device copies (copy-in stream) overlap
        # step i-1's compute and step i-2's device->host copies (copy-out
        # stream), as a serving or training loop feeding from pinned host
        # memory would run.  Two device input sets; a set is rewritten only
        # after the compute that read it has finished.
        comp = torch.cuda.current_stream(dev)
        cin = torch.cuda.Stream(dev)
        cout = torch.cuda.Stream(dev)
        bufs = [[torch.empty_like(q.detach()) for _ in range(4)] for _ in range(2)]
        free_ev = [None, None]

        def e2e_step(i):
            sset = bufs[i % 2]
            with torch.cuda.stream(cin):
                if free_ev[i % 2] is not None:
                    cin.wait_event(free_ev[i % 2])
                for b, hsrc in zip(sset, (hq, hk, hv, hdo)):
                    b.copy_(hsrc, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(cin)
            comp.wait_event(ready)
            qi, ki, vi = (b.detach().requires_grad_(True) for b in sset[:3])
            out = varlen_attention_triton_autograd(qi, ki, vi, cu, causal=causal)
            out.backward(sset[3])
            done = torch.cuda.Event()
            done.record(comp)
            free_ev[i % 2] = done
            with torch.cuda.stream(cout):
                cout.wait_event(done)
                for hdst, t in zip((ho, hdq, hdk, hdv), (out.detach(), qi.grad, ki.grad, vi.grad)):
                    hdst.copy_(t, non_blocking=True)
                    t.record_stream(cout)

        e2e_step(0)
        e2e_step(1)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        cin.wait_stream(comp)  # the first copy starts inside the timed region
        for i in range(args.e2e_steps):
            e2e_step(i)
        comp.wait_stream(cout)  # ... and the last copy back ends inside it
        e1.record(comp)
        torch.cuda.synchronize()
        e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e_step = float(e_ms[0]) / args.e2e_steps
        nbytes = int(total_T) * H * D * q.element_size()  # one (T, H, D) tensor, all ranks
        e2e = {
            "value": total_T / (e_step / 1e3),
            "unit": "tokens/s",
            "ms_per_step": e_step,
            "h2d_bytes_per_step": int(4 * nbytes),  # q, k, v, dO
            "d2h_bytes_per_step": int(4 * nbytes),  # out, dq, dk, dv
            "path": "varlen_attention_triton_autograd with pinned host q/k/v/dO in, out/dq/dk/dv back to pinned host; copies in, compute and copies out of consecutive steps overlap on three streams",
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, sample = cpu_reference_rate(lengths, H, D, causal)
        cpu = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16" if args.dtype_name == "float16" else "bf16",
            "data": "synthetic",
            "config": workload_config(args, lengths, H, D, causal, world),
            "tflops": tflops,
            "tflops_frac_of_peak": tflops / (peak_tf * world),
            "roofline": {
                "kernel": "attn_bwd_kernel<128, bf16, causal> (dK/dV/dQ, 10*H*D*pairs FLOPs)",
                "bound": "tensor",
                "achieved": ach_bwd,
                "peak": peak_tf,
                "unit": "TFLOP/s",
                "frac": ach_bwd / peak_tf,
                "peak_source": f"{peak_kind} bf16_tflops_sustained (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback 1.4 PFLOP/s sustained",
                "traffic": traffic,
                "avg_launch_ms": bwd_avg_ms,
            },
            "kernels": {
                "attn_fwd": {"avg_ms": fwd_avg_ms, "launches": nf, "tflops": ach_fwd, "frac": ach_fwd / peak_tf},
                "attn_bwd": {"avg_ms": bwd_avg_ms, "launches": nb, "tflops": ach_bwd, "frac": ach_bwd / peak_tf},
            },
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(total_launch),
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
