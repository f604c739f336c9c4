#!/usr/bin/env python
"""Varlen attention fwd+bwd throughput of scree_b200 on B200 (one JSON line).

    python bench.py [--gpus N --steps K --warmup W] [--impl native|reference]

Workload (default): cfg4 — 64 sequences, lengths lognormal(ln 2048, 0.6) clipped
to [16, 16384] at seed 0 (T = 158,330 tokens), q/k/v/dO ~ N(0,1) bf16 of shape
(T, 32 heads, 128), causal.  A step is one forward + backward through the
drop-in autograd entry point (varlen_attention_triton_autograd -> out.backward).

Timing, identical at every N: each timed step has its own CUDA-event pair on
the compute stream, and a 256 MB buffer (twice the 126 MB L2) is written
before every step, outside its events; the step times are summed.

Multi-GPU (torchrun, one process per GPU): the fixed batch is split by whole
sequences, longest-processing-time-first on L^2, identically on every rank (the
plan is broadcast from rank 0 over NCCL and checked).  ``value`` is the
compute-only throughput (every rank keeps its outputs, as a data-parallel rank
does): all tokens / the max over ranks of the step time ("strong" scaling:
total work fixed).  ``with_gather`` adds the exchange of the per-rank outputs
(O, dQ, dK, dV) to rank 0 by NCCL send/recv inside every step and reports that
time too.

At N=1 the same line also carries ``norms``: cfg3 RMSNorm / LayerNorm forward
and backward, varlen softmax and the pack / to_padded / from_padded gathers,
each timed per launch with CUDA events (L2 flushed before each), as GB/s of
algorithmic bytes and as a fraction of the measured HBM bandwidth.

--impl reference times the reference algorithm on the host CPU instead: the
numpy oracle (a restatement of scree.kernels.reference; the reference itself is
pure Python and is not installed on the GPU box), fp32, all host threads.  Each
step processes one of the 32 heads of every cfg4 sequence (heads are
independent and cost the same); the value is scaled by the head count.
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
CLOCK_PERIOD_S = 0.05


TRAFFIC_FILE = ROOT / "profiles" / "attn_bwd_small_traffic.json"


def scaled_traffic(groups, D, causal):
    """DRAM bytes per backward launch for this rank's workload, scaled from one
    ncu capture of dram__bytes_read.sum + dram__bytes_write.sum on a small case
    (TRAFFIC_FILE) by the ratio of causal pairs x heads (the backward's traffic
    grows with the (key tile, query tile) pairs: Q/dO re-reads and the fp32 dQ
    accumulation).  Returns (bytes or None, description)."""
    from scree_b200 import workloads

    if not TRAFFIC_FILE.exists():
        return None, "no capture"
    try:
        d = json.loads(TRAFFIC_FILE.read_text())
        units_small = float(d["pairs_x_heads"])
        units = float(sum((workloads.causal_pairs(ls) if causal else sum(L * L for L in ls)) * hs
                          for hs, ls in groups))
        if d.get("head_dim") != D:
            return None, "capture has another head_dim"
        scale = units / units_small
        return float(d["bytes_per_launch"]) * scale, (
            f"{d['bytes_per_launch'] / 1e9:.3f} GB per launch measured by ncu on {d['case']} "
            f"({TRAFFIC_FILE.name}), scaled x{scale:.2f} by causal pairs x heads")
    except Exception as e:  # malformed file: report, do not guess
        return None, f"unreadable capture: {e}"


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
    """Samples SM clock and clock-event reasons every 50 ms through NVML (read only)."""

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
            self._stop.wait(CLOCK_PERIOD_S)

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
def _cpu_threads():
    """Host threads for the numpy oracle, with BLAS / OpenMP pools raised to
    all of them (torchrun sets OMP_NUM_THREADS=1 for its ranks)."""
    cores = len(os.sched_getaffinity(0))
    try:
        import threadpoolctl

        threadpoolctl.threadpool_limits(cores)
    except Exception:
        pass
    return cores


def _cpu_head_step(lengths, H, D, causal, head, seed=0, fwd_only=False):
    """One step of the CPU sample: the numpy oracle's fwd+bwd (fp32; the
    forward alone with `fwd_only`) on head `head` of every sequence of the
    workload.  Inputs are drawn per head from a seeded generator (N(0,1), as on
    the GPU)."""
    import oracle

    rng = np.random.default_rng(seed + head)
    offs = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    T = int(offs[-1])
    q, k, v, do = (rng.standard_normal((T, 1, D), dtype=np.float32) for _ in range(4))
    t0 = time.perf_counter()
    oracle.attention_fwd(q, k, v, offs, causal=causal, dtype=np.float32)
    if not fwd_only:
        oracle.attention_bwd(do, q, k, v, offs, causal=causal, dtype=np.float32)
    return time.perf_counter() - t0


def cpu_reference_rate(lengths, H, D, causal, repeats=2, fwd_only=False):
    """CPU baseline for the GPU line: the oracle on one head of every sequence,
    `repeats` times (about 10-20 s); tokens/s = T / (H x median head time)."""
    cores = _cpu_threads()
    times = [_cpu_head_step(lengths, H, D, causal, head=h, fwd_only=fwd_only) for h in range(repeats)]
    t = statistics.median(times)
    T = sum(lengths)
    rate = T / (t * H)
    sample = (f"numpy oracle (restatement of scree.kernels.reference) fp32 {'forward' if fwd_only else 'fwd+bwd'} of 1 of {H} heads "
              f"over all {len(lengths)} sequences (T={T}, D={D}), median of {len(times)} heads = {t:.2f} s; "
              f"x{H} heads (independent, identical cost) for the whole workload")
    return rate, cores, sample


def run_reference_arm(args, lengths, H, D, causal):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cores = _cpu_threads()
    fo = getattr(args, "fwd_only", False)
    for i in range(args.warmup):
        _cpu_head_step(lengths, H, D, causal, head=i % H, fwd_only=fo)
    times = [_cpu_head_step(lengths, H, D, causal, head=i % H, fwd_only=fo) for i in range(args.steps)]
    dt = sum(times) / len(times)
    T_total = sum(lengths)
    value = T_total / (dt * H)
    sample = (f"each step: numpy oracle (restatement of scree.kernels.reference) fp32 {'forward' if fo else 'fwd+bwd'} of one of "
              f"the {H} heads (rotating) over all {len(lengths)} sequences (T={T_total}, D={D}) on {cores} "
              f"host threads, {dt:.2f} s per head; value = T / ({H} x that time): heads are independent "
              f"and cost the same")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "ms_per_step_note": "time of one step of the sample (one head of every sequence)",
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(args, lengths, H, D, causal, world),
        "tflops": workloads_flops(lengths, 1, D, causal, fwd_only=fo) / dt / 1e12,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workloads_flops(lengths, H, D, causal, fwd_only=False):
    from scree_b200 import workloads

    return workloads.attn_flops(lengths, H, D, causal, fwd=True, bwd=not fwd_only)


_LEN_DESC = {
    "cfg2": "lognormal(ln 700, 0.6) rescaled to 12160 tokens",
    "cfg4": "lognormal(ln 2048, 0.6) clip [16,16384]",
    "cfg5": "lognormal(ln 1024, 1.2) clip [1,32768], 4 forced length-1",
}


def workload_config(args, lengths, H, D, causal, world):
    return {
        "workload": f"{args.config}: {len(lengths)} seqs {_LEN_DESC[args.config]} seed 0, "
        f"T={sum(lengths)}, H={H}, D={D}, {getattr(args, 'dtype_name', 'bfloat16')}, {'causal' if causal else 'non-causal'} "
        f"{'forward only' if getattr(args, 'fwd_only', False) else 'fwd+bwd'}",
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
def measure_norms(steps, warmup, with_cpu=True):
    """cfg3: 64 sequences, lengths lognormal(ln 256, 0.6) (T = 19,794), hidden 4096
    bf16.  Each op is timed per launch with CUDA events; a 256 MB buffer is
    written between launches to flush the 126 MB L2.  Bandwidth = algorithmic
    bytes (reads + writes the op must do) / time, against MEASURED_PEAKS hbm_gbs.
    Returns (per-op results, cpu baseline or None, hbm peak, peak source, T)."""
    import torch

    import scree_b200 as scree
    from scree_b200 import _lib, workloads
    from scree_b200.kernels import native

    dev = torch.device("cuda", torch.cuda.current_device())
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
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
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
        for _ in range(max(3, warmup)):
            fn()
        # Kernel-only time from the library's CUDA-event hooks around each
        # launch (all launches of one call summed); the 256 MB flush is written
        # before every call.  The softmax kernels report under the norm fwd /
        # bwd event kinds.
        kind_ = _lib.PROF_NORM_FWD if name.endswith("_fwd") else (_lib.PROF_NORM_BWD if name.endswith("_bwd") else _lib.PROF_GATHER)
        times = []
        _lib.profile_read(kind_)
        _lib.profile_enable(True)
        for _ in range(steps):
            flush.fill_(1)
            fn()
            torch.cuda.synchronize()
            tms, _nl = _lib.profile_read(kind_)
            times.append(tms)
        _lib.profile_enable(False)
        ms = statistics.median(times)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"ms": ms, "algorithmic_bytes": int(nbytes), "gb_s": gbs, "frac": gbs / hbm}
    assert _lib.device_status() == 0
    cpu = None
    if with_cpu:
        import oracle

        cores = _cpu_threads()
        xn = x.float().cpu().numpy()
        wn = w.cpu().numpy()
        oracle.rmsnorm_fwd(xn, wn, 1e-5, dtype=np.float32)
        t0 = time.perf_counter()
        oracle.rmsnorm_fwd(xn, wn, 1e-5, dtype=np.float32)
        t_cpu = time.perf_counter() - t0
        cpu = {"value": 2 * T * C * b / t_cpu / 1e9, "unit": "GB/s", "cores": cores,
               "kind": "port", "sample": f"rmsnorm_fwd on the full cfg3 batch (fp32 numpy oracle), {t_cpu:.3f} s"}
    return res, cpu, hbm, kind, T


def measure_prenorm_qkv(steps, warmup):
    """Fused RMSNorm -> QKV projection on cfg3's rows (T = 19,794, hidden 4096, bf16)
    with a (4096, 3 x 4096) weight: 2 T C N FLOPs per call, timed per launch with
    CUDA events (L2 flushed before each) against the burst bf16 GEMM peak."""
    import torch

    from scree_b200 import _lib, workloads
    from scree_b200.kernels import native

    dev = torch.device("cuda", torch.cuda.current_device())
    T, C, N = sum(workloads.cfg3_lengths()), 4096, 3 * 4096
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((T, C), device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn((C, N), device=dev, generator=g) / 64).to(torch.bfloat16)
    gamma = 1 + 0.02 * torch.randn(C, device=dev, generator=g)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(max(3, warmup)):
        native.rmsnorm_qkv(x, gamma, w, 1e-6)
    times = []
    _lib.profile_read(_lib.PROF_NORM_FWD)
    _lib.profile_enable(True)
    for _ in range(steps):
        flush.fill_(1)
        native.rmsnorm_qkv(x, gamma, w, 1e-6)
        torch.cuda.synchronize()
        times.append(_lib.profile_read(_lib.PROF_NORM_FWD)[0])
    _lib.profile_enable(False)
    ms = statistics.median(times)
    peaks, kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tf = 2.0 * T * C * N / (ms / 1e3) / 1e12
    return {"workload": f"x ({T}, {C}) bf16 (cfg3 rows), Wqkv ({C}, {N}), gamma fp32; y = rmsnorm(x) * gamma @ Wqkv",
            "ms": ms, "tflops": tf, "frac": tf / peak, "peak_tflops": peak,
            "peak_source": f"{kind} bf16_tflops (burst)", "note": "GEMM kernel time; the row-statistics pass (T x C read) and the gamma-folding pass over the weight (C x N) are separate launches"}


def run_norm_suite(args):
    import torch

    torch.cuda.set_device(0)
    res, cpu, hbm, kind, T = measure_norms(args.steps, args.warmup, not args.no_cpu_baseline)
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
        "config": {"workload": f"cfg3: 64 seqs lognormal(ln 256, 0.6) seed 0, T={T}, hidden 4096 bf16",
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
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--config", default="cfg4", choices=["cfg4", "cfg2", "cfg5"])
    ap.add_argument("--e2e-steps", type=int, default=16,
                    help="pipelined end-to-end steps timed (the first copy-in and last copy-out are not overlapped)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-norms", action="store_true", help="skip the cfg3 norms/softmax/gathers object")
    ap.add_argument("--no-gather", action="store_true", help="N>1: skip the with-output-exchange timing")
    ap.add_argument("--non-causal", action="store_true")
    ap.add_argument("--fwd-only", action="store_true",
                    help="time the forward alone (inference; cfg5 is specified forward only)")
    ap.add_argument("--shard", choices=["seqs", "heads"], default="seqs",
                    help="multi-GPU split: whole sequences (default) or sequences split by head groups")
    ap.add_argument("--suite", choices=["attention", "norms", "qkv"], default="attention",
                    help="norms: cfg3 RMSNorm/LayerNorm fwd+bwd and pack/unpack/to_padded/from_padded; "
                         "qkv: the fused RMSNorm -> QKV projection alone")
    ap.add_argument("--max-seqs", type=int, default=0, help="keep only the first N sequences (small profiling case)")
    args = ap.parse_args()

    from scree_b200 import workloads

    if args.suite == "norms":
        run_norm_suite(args)
        return
    if args.suite == "qkv":
        import torch

        torch.cuda.set_device(0)
        print(json.dumps({"suite": "qkv", "steps": args.steps, "warmup": max(3, args.warmup),
                          "prenorm_qkv": measure_prenorm_qkv(args.steps, args.warmup)}), flush=True)
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
        # (sequence, head group) units, split as finely as the balance needs;
        # every (sequence, head) of a rank's units is laid out as its own packed
        # single-head sequence, so the rank runs ONE attention call (H = 1) over
        # all of them whatever their head counts (heads are independent).
        plan = shard.plan_units(lengths, world, H, max_groups=H)
        if world > 1:
            plan = shard.broadcast_plan(plan)
        groups = [(1, [lengths[u.seq] for u in plan[rank] for _ in range(u.heads)])]
        args.no_e2e = True  # the end-to-end path is measured on whole sequences
        args.no_gather = True
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

    from scree_b200.kernels.native import varlen_attention_triton

    def step():
        for qg, kg, vg, dog, cug in calls:
            if args.fwd_only:
                varlen_attention_triton(qg.detach(), kg.detach(), vg.detach(), cug, causal=causal)
                continue
            for t in (qg, kg, vg):
                t.grad = None
            out = varlen_attention_triton_autograd(qg, kg, vg, cug, causal=causal)
            out.backward(dog)

    tensor_bytes = sum(qg.numel() for qg, *_ in calls) * q.element_size()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    args.l2_note = (f"q/k/v/dO {tensor_bytes / 1e6:.0f} MB each per rank; a 256 MB buffer is written "
                    f"before every timed step, outside its CUDA events (same at every N)")

    def timed_steps(n, fn):
        """Sum of per-step CUDA-event times of n steps, L2 flushed before each."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for a, b in evs:
            flush.fill_(1)
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs)

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
    elapsed_ms = timed_steps(args.steps, step)
    launches = _lib.launch_count() - n0
    _lib.profile_enable(False)
    fwd_ms, nf = _lib.profile_read(_lib.PROF_ATTN_FWD)
    bwd_ms, nb = _lib.profile_read(_lib.PROF_ATTN_BWD)
    if world > 1:
        dist.barrier()
    sampler.stop()
    assert _lib.device_status() == 0, "kernel reported an error (device status word)"

    # ------------------------------------------------------------ with output exchange
    with_gather = None
    if world > 1 and args.shard == "seqs" and not args.no_gather:
        offs_g = np.concatenate([[0], np.cumsum(lengths)])
        mine = shard.local_shard(offs_g, plan, rank)
        T_all = int(offs_g[-1])
        gplan = shard.GatherPlan(plan, offs_g, rank, dev)

        pending = []  # the previous step's transfer and the tensors it reads

        def step_gather():
            # Step i's outputs travel while step i+1 computes; its requests are
            # waited on after step i+1 is enqueued.
            if args.fwd_only:
                sent = [varlen_attention_triton(q.detach(), k.detach(), v.detach(), cu, causal=causal)]
            else:
                for t in (q, k, v):
                    t.grad = None
                out = varlen_attention_triton_autograd(q, k, v, cu, causal=causal)
                out.backward(do)
                sent = [out.detach(), q.grad, k.grad, v.grad]
            _, reqs = gplan.run(sent, defer=True)
            for r in (pending.pop()[0] if pending else []):
                r.wait()
            pending.append((reqs, sent))

        def drain():
            for r in (pending.pop()[0] if pending else []):
                r.wait()

        for _ in range(2):
            step_gather()
        drain()
        torch.cuda.synchronize()
        dist.barrier()
        g_steps = max(3, min(args.steps, 20))
        # One event pair over all steps (the transfers overlap the next step's
        # compute, so per-step pairs would split them); no L2 flush: each rank's
        # inputs are larger than L2 at cfg4 up to 8 GPUs.
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(g_steps):
            step_gather()
        drain()
        g1.record()
        torch.cuda.synchronize()
        g_ms = g0.elapsed_time(g1)
        gm = torch.tensor([g_ms / g_steps], dtype=torch.float64, device=dev)
        dist.all_reduce(gm, op=dist.ReduceOp.MAX)
        recv_bytes = (1 if args.fwd_only else 4) * (T_all - mine.tokens) * H * D * q.element_size()
        with_gather = {
            "ms_per_step": float(gm[0]),
            "steps": g_steps,
            "value": float(sum(lengths)) / (float(gm[0]) / 1e3),
            "unit": "tokens/s",
            "collective": (f"NCCL send/recv to rank 0 of every rank's {'O' if args.fwd_only else 'O, dQ, dK, dV'} rows, one message per sequence and tensor straight into rank 0's global-order outputs, one batch per step (NVLink), overlapping the next step's compute"),
            "timing": "one CUDA-event pair over all steps on the compute stream, max over ranks, last transfer included",
            "bytes_into_rank0_per_step": int(recv_bytes),
        }

    flops_mine = sum(workloads.attn_flops(ls, hs, D, causal, fwd=True, bwd=not args.fwd_only) for hs, ls in groups)
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
    # Denominator by the clock record of the timed region: the burst GEMM figure
    # when the SM clock stayed at its maximum with no power capping, else the
    # sustained figure (measured as a seconds-long loop under the power cap).
    # Both fractions are reported.
    clk = sampler.summary()
    capped = ("sw_power_cap" in clk["reasons"]) or (
        clk["sm_mhz"] is not None and clk["sm_max_mhz"] and clk["sm_mhz"] < 0.95 * clk["sm_max_mhz"])
    peak_burst = float(peaks.get("bf16_tflops", peaks.get("bf16_tflops_sustained")))
    peak_sus = float(peaks.get("bf16_tflops_sustained", peak_burst))
    peak_tf = peak_sus if capped else peak_burst
    peak_name = "bf16_tflops_sustained" if capped else "bf16_tflops (burst)"
    bwd_avg_ms = bwd_ms / max(nb, 1)
    fwd_avg_ms = fwd_ms / max(nf, 1)
    # This rank's FLOPs per step over its kernel time per step (one launch per
    # step and kind, or one per head-count group with --shard heads).
    ach_bwd = flops_bwd_mine / (bwd_ms / args.steps / 1e3) / 1e12 if bwd_ms > 0 else 0.0
    ach_fwd = flops_fwd_mine / (fwd_ms / args.steps / 1e3) / 1e12 if fwd_ms > 0 else 0.0
    ach_top = ach_fwd if args.fwd_only else ach_bwd  # the dominant kernel of the step
    if args.fwd_only:
        traffic, traffic_src = None, "no DRAM capture of the forward kernel at this size"
    else:
        traffic, traffic_src = scaled_traffic(groups, D, causal)

    # ------------------------------------------------------------ end to end
    e2e = None
    if not args.no_e2e:
        n_in = 3 if args.fwd_only else 4  # q, k, v (, dO) in; out (, dq, dk, dv) back
        n_out = 1 if args.fwd_only else 4
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
                for b, hsrc in list(zip(sset, (hq, hk, hv, hdo)))[:n_in]:
                    b.copy_(hsrc, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(cin)
            comp.wait_event(ready)
            if args.fwd_only:
                out = varlen_attention_triton(sset[0], sset[1], sset[2], cu, causal=causal)
                results = (out,)
            else:
                qi, ki, vi = (b.detach().requires_grad_(True) for b in sset[:3])
                out = varlen_attention_triton_autograd(qi, ki, vi, cu, causal=causal)
                out.backward(sset[3])
                results = (out.detach(), qi.grad, ki.grad, vi.grad)
            done = torch.cuda.Event()
            done.record(comp)
            free_ev[i % 2] = done
            with torch.cuda.stream(cout):
                cout.wait_event(done)
                for hdst, t in zip((ho, hdq, hdk, hdv), results):
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
            "h2d_bytes_per_step": int(n_in * nbytes),  # q, k, v (, dO)
            "d2h_bytes_per_step": int(n_out * nbytes),  # out (, dq, dk, dv)
            "path": ("varlen_attention_triton with pinned host q/k/v in, out back to pinned host"
                     if args.fwd_only else
                     "varlen_attention_triton_autograd with pinned host q/k/v/dO in, out/dq/dk/dv back to pinned host")
            + "; copies in, compute and copies out of consecutive steps overlap on three streams",
        }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, sample = cpu_reference_rate(lengths, H, D, causal, fwd_only=args.fwd_only)
        cpu = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}

    norms = None
    prenorm_qkv = None
    if world == 1 and not args.no_norms:
        nres, ncpu, hbm, nkind, nT = measure_norms(max(10, min(args.steps, 30)), args.warmup, not args.no_cpu_baseline)
        norms = {
            "workload": f"cfg3: 64 seqs lognormal(ln 256, 0.6) seed 0, T={nT}, hidden 4096 bf16; L2 flushed before each launch",
            "hbm_peak_gbs": hbm,
            "peak_source": f"{nkind} hbm_gbs",
            "ops": {k_: {"gb_s": round(v_["gb_s"], 1), "frac": round(v_["frac"], 4), "ms": v_["ms"],
                         "algorithmic_bytes": v_["algorithmic_bytes"]} for k_, v_ in nres.items()},
            "cpu_baseline": ncpu,
        }
        prenorm_qkv = measure_prenorm_qkv(max(10, min(args.steps, 30)), args.warmup)
    else:
        prenorm_qkv = None

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
            "tflops_frac_of_burst_peak": tflops / (peak_burst * world),
            "tflops_frac_of_sustained_peak": tflops / (peak_sus * world),
            "roofline": {
                "kernel": (f"attn_fwd_kernel<{D}, {'causal' if causal else 'full'}> (4*H*D*pairs FLOPs)" if args.fwd_only
                           else f"attn_bwd_kernel<{D}, {'causal' if causal else 'full'}> (dK/dV/dQ, 10*H*D*pairs FLOPs)"),
                "bound": "tensor",
                "achieved": ach_top,
                "peak": peak_tf,
                "unit": "TFLOP/s",
                "frac": ach_top / peak_tf,
                "frac_of_burst_peak": ach_top / peak_burst,
                "frac_of_sustained_peak": ach_top / peak_sus,
                "peak_source": (f"{peak_kind} {peak_name} (MEASURED_PEAKS.json), chosen by the clock record "
                                f"({'power-capped' if capped else 'unthrottled'})" if peak_kind == "measured"
                                else "fallback (1.59 PFLOP/s burst, 1.4 sustained)"),
                "traffic": traffic,
                "traffic_source": traffic_src,
                "avg_launch_ms": fwd_avg_ms if args.fwd_only else bwd_avg_ms,
            },
            "kernels": {
                "attn_fwd": {"avg_ms": fwd_avg_ms, "launches": nf, "tflops": ach_fwd, "frac": ach_fwd / peak_tf},
                "attn_bwd": {"avg_ms": bwd_avg_ms, "launches": nb, "tflops": ach_bwd, "frac": ach_bwd / peak_tf},
            },
            "compute_only_ms": ms_step,
            "with_gather": with_gather,
            "norms": norms,
            "prenorm_qkv": prenorm_qkv,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(total_launch),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
