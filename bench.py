#!/usr/bin/env python3
"""Benchmark of the variable-K grouped FP8 wgrad on 1..8 B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config gate_up] [--impl ours|reference]

One step = one call of the hot path over one synthetic batch: every expert's weight gradient
C[g] = sL*sR * LHS_g^T RHS_g for the configured problem (default: the gate_up benchmark,
GPT-OSS-20B gate_up_wgrad: G=32, M_total=131072, 2880 x 5760, e4m3 x e5m2 -> bf16).
Metric: TFLOPS = 2*M_total*OUT_M*OUT_N / time (launcher.cpp:76), whole job over all GPUs.

N > 1 (launched by torchrun): expert-sharded weak scaling. Every rank owns its own
gate_up-shaped shard (32 experts, 131072 tokens, 2880 x 5760) of a 32N-expert problem and runs
the kernel on it; there is no collective on the timed path (the barrier and the max-over-ranks
reduction sit outside the timed region). ``--config shard120b`` instead partitions the
GPT-OSS-120B-shaped problem (G=128, M_total=1048576) contiguously across the N ranks.

Timing: W untimed warm-up steps, then K steps between CUDA events on the launching stream,
bracketed by a barrier and torch.cuda.synchronize(); the time is the max over ranks. The
operands (1.13 GB for gate_up) are far larger than the 126 MB L2, so no L2 flush is needed.

Other legs (one GPU; not the driver's line): --op quantize (the producer step: per-expert amax +
fp8 quantisation of x and dy, GB/s), --op fwd --site <site> (the fixed-K grouped GEMM of a
forward / data-gradient site, TFLOPS, with cuBLAS per expert beside it), --op layer (one training
step of the FP8 MoE linear layer).

Beside the headline the line carries ``other_workloads``: at N = 1 the down_wgrad and skewed-
routing problems, and at every N the GPT-OSS-120B-shaped problem (G = 128, M_total = 1048576)
split into contiguous expert ranges across the ranks (strong scaling; max over ranks, with the
per-rank times and token counts).

--impl reference: the reference's own implementation of the path cannot run here (AMD gfx950
code object + a Triton kernel from the absent primus_turbo package), so the reference arm
times the CPU restatement of its algorithm (oracle/, torch fp32 dequantise + matmul per expert)
on all host threads, rank 0 only. One step multiplies the first quarter of every expert's tokens
(all experts, in proportion), the same sample the repo arm's ``cpu_baseline`` times, and the
line carries the same metric string as the repo arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF_PUBLISHED_TFLOPS = 1237.0  # MI355X, hand-optimised ASM, gate_up_wgrad (README.md:60)
FP8_NOMINAL_TFLOPS = 4500.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="gate_up",
                    choices=["gate_up", "down", "skew", "shard120b", "ref_exp"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="wgrad", choices=["wgrad", "quantize", "fwd", "layer"],
                    help="wgrad: the grouped GEMM (default, the headline); quantize: the producer "
                         "step (per-expert amax + fp8 quantisation of x and dy) at the same shape; "
                         "fwd: the fixed-K grouped GEMM of a forward/data-gradient site (--site); "
                         "layer: one forward + backward step of the FP8 MoE linear layer")
    ap.add_argument("--site", default="gate_up_fwd",
                    choices=["gate_up_fwd", "down_fwd", "down_dgrad", "gate_up_dgrad"],
                    help="call site of --op fwd (bench.py:154-181 of the reference harness)")
    ap.add_argument("--no-cublas", action="store_true", help="--op fwd: skip the cuBLAS leg")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-other", action="store_true",
                    help="skip the down / skew / 120B-split workloads printed beside the headline")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="approximate CPU-baseline sample budget")
    ap.add_argument("--groups", type=int, default=None,
                    help="override G (smaller cases for profiling; not a bench line)")
    ap.add_argument("--tokens", type=int, default=None,
                    help="override M_total (smaller cases for profiling; not a bench line)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_peaks():
    """(fp8 dense peak TFLOP/s, hbm GB/s, description). FP8 = 2x the measured bf16 cuBLAS burst
    figure (the B200 tensor core runs fp8 at twice the bf16 rate)."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return (2.0 * float(d["bf16_tflops"]), float(d["hbm_gbs"]),
                "of measured: 2 x MEASURED_PEAKS.json bf16_tflops (cuBLAS bf16 burst)")
    return 2.0 * 1590.0, 6650.0, "of fallback: 2 x 1.59 PFLOP/s bf16"


def profile_traffic(workload: str):
    """dram bytes per launch of the dominant kernel from the committed ncu summary, or None."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None
    d = json.loads(f.read_text())
    ent = d.get(workload)
    return None if ent is None else float(ent["dram_bytes_per_launch"])


class ClockSampler:
    """Polls NVML (SM clock, power, clock-event reasons) every `period` seconds in a thread.
    `window(t0, t1)` summarises the samples taken between two host timestamps. NVML averages
    each reading over its own sample period (1/6 s to 1 s), so a short timed region yields few
    and partly averaged samples; `sustained()` reads a longer untimed stretch of the same work."""

    NAMES = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
             "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int, period: float = 0.005):
        import threading

        self.samples = []  # (t, sm_mhz, power_w, reasons_mask)
        self.period = period
        self.stop_ev = threading.Event()
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml

            self.nvml = pynvml
            self.handle = torch.cuda._get_pynvml_handler(device)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:  # NVML unavailable: report that instead of guessing
            self.handle = None
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nvml
        while not self.stop_ev.is_set():
            try:
                self.samples.append((time.perf_counter(),
                                     float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)),
                                     nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0,
                                     int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle))))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop_ev.set()
        if self.handle is not None:
            self.thread.join(timeout=5)

    def window(self, t0: float, t1: float) -> dict:
        if self.handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        sel = [s for s in self.samples if t0 <= s[0] <= t1]
        if not sel:  # region shorter than the polling period: nearest sample after it
            later = [s for s in self.samples if s[0] >= t0]
            sel = later[:1]
        reasons = sorted(n for n, bit in self.NAMES.items() if any(s[3] & bit for s in sel))
        return {"sm_mhz": statistics.median(s[1] for s in sel) if sel else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(sel),
                "power_w_max": max((s[2] for s in sel), default=None), "source": "nvml"}


def build_problem(args, rank, world, device):
    from ggemm_asm_b200 import inputs, sharding

    if args.config == "shard120b":
        lens = inputs.config_lens("shard120b", args.seed)
        shards = sharding.partition(lens, world)
        sh = shards[rank]
        full = inputs.offsets_from_lens(lens)
        p = inputs.make_problem("shard120b", seed=args.seed, device=device, lens=lens,
                                rows=(sh.t_begin, sh.t_end))
        loc = sharding.local_offsets(full, sh)
        return inputs.Problem(
            name=f"shard120b[{sh.g_begin}:{sh.g_end}]", G=sh.groups, M_total=sh.tokens,
            OUT_M=p.OUT_M, OUT_N=p.OUT_N, lens=lens[sh.g_begin:sh.g_end], offs=loc,
            lhs=p.lhs, rhs=p.rhs, lhs_scale=p.lhs_scale, rhs_scale=p.rhs_scale,
            group_offs=torch.from_numpy(loc.copy()).to(device)), "strong"
    name = {"ref_exp": "gate_up"}.get(args.config, args.config)
    seed = args.seed + 1000 * rank  # each rank owns a distinct shard of the 32N-expert job
    if args.config == "ref_exp":
        lens = inputs.reference_exponential_lens(32, 131072, 42)
        p = inputs.make_problem("gate_up", seed=seed, device=device, lens=lens)
    elif args.groups is not None or args.tokens is not None:
        cfg = inputs.CONFIGS[name]
        p = inputs.make_problem(name, seed=seed, device=device, G=args.groups or cfg["G"],
                                M_total=args.tokens or cfg["M_total"])
    else:
        p = inputs.make_problem(name, seed=seed, device=device)
    return p, "weak"


def workload_name(config: str) -> str:
    """The wgrad workload a config measures (shard120b and ref_exp are gate_up-shaped)."""
    return "gate_up" if config in ("gate_up", "ref_exp", "shard120b") else config


def metric_name(config: str) -> str:
    """The metric string both arms print for a config (the driver compares them verbatim)."""
    return f"{workload_name(config)}_wgrad FP8 TFLOPS (whole job)"


# Fraction of every expert's tokens that one CPU sample step multiplies: all experts, in
# proportion to their sizes, so the sample has the workload's expert mix (about 0.6 s of
# 16-thread CPU time at the gate_up shape).
CPU_SAMPLE_FRAC = 0.25


def cpu_sample_step(p_cpu, frac: float = CPU_SAMPLE_FRAC) -> float:
    """One step of the CPU restatement (oracle/, torch CPU fp32 dequantise + matmul) over the
    first ceil(frac * K_g) tokens of every expert g; returns the FLOPs done."""
    from oracle import vark_oracle as vo

    offs = p_cpu.group_offs.clone()
    flops = 0.0
    for g in range(p_cpu.G):
        k = int(np.ceil(frac * float(p_cpu.lens[g])))
        if k == 0:
            continue
        sub = offs.clone()
        sub[g + 1] = offs[g] + k  # the oracle reads only [offs[g], offs[g+1]) for group g
        vo.wgrad_torch(p_cpu.lhs, p_cpu.rhs, p_cpu.lhs_scale, p_cpu.rhs_scale, sub, groups=[g])
        flops += 2.0 * k * p_cpu.OUT_M * p_cpu.OUT_N
    return flops


def cpu_sample_desc(p_cpu, frac: float = CPU_SAMPLE_FRAC) -> str:
    return (f"every step: the first {frac:.0%} of every expert's tokens ({p_cpu.G} experts, "
            f"{int(np.ceil(frac * p_cpu.lens).sum())} of {int(p_cpu.lens.sum())} tokens) of the "
            f"same problem, torch CPU fp32 dequantise + matmul per expert")


def cpu_oracle_rate(p_cpu, budget_s: float):
    """Time the CPU sample steps until `budget_s` has passed; returns (TFLOPS, sample, secs)."""
    done_flops, t_total, steps = 0.0, 0.0, 0
    while t_total < budget_s:
        t0 = time.perf_counter()
        done_flops += cpu_sample_step(p_cpu)
        t_total += time.perf_counter() - t0
        steps += 1
    return done_flops / t_total / 1e12, f"{steps} steps; " + cpu_sample_desc(p_cpu), t_total


def run_reference(args):
    """Reference arm: the CPU restatement of the reference algorithm, rank 0 only."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    # The problem the repo arm's rank 0 runs for this config (routing, shape, --groups/--tokens),
    # generated on the host: ref_exp keeps the reference's exponential routing, shard120b is the
    # whole 120B-shaped problem.
    p, _ = build_problem(args, 0, 1, "cpu")
    for _ in range(args.warmup):
        cpu_sample_step(p)
    flops, t = 0.0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        flops += cpu_sample_step(p)
        t += time.perf_counter() - t0
    v = flops / t / 1e12
    cores = torch.get_num_threads()
    sample = cpu_sample_desc(p)
    line = {"impl": "reference", "metric": metric_name(args.config),
            "value": v, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config}_wgrad", "G": p.G, "M_total": p.M_total,
                       "OUT_M": p.OUT_M, "OUT_N": p.OUT_N},
            "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference kernel unavailable here (AMD gfx950 code object; primus_turbo "
                    "Triton oracle absent); timed its algorithm restated on the CPU (oracle/)"}
    print(json.dumps(line), flush=True)


def run_quantize(args):
    """Producer step at the gate_up shape, one GPU: per step, quantise x [M_total, 2880] bf16 ->
    e4m3 and dy [M_total, 5760] bf16 -> e5m2 with one scale per expert (two launches). Metric:
    algorithmic HBM bytes per second (2 B read + 1 B written per element; scales and offsets
    are negligible), against the measured copy bandwidth."""
    from ggemm_asm_b200 import _lib, inputs, quantize_fp8

    rank, world, local = dist_env()
    if world != 1:
        raise SystemExit("--op quantize runs on one GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    cfg = inputs.CONFIGS["gate_up"]
    lens = inputs.config_lens("gate_up", args.seed)
    if args.groups is not None or args.tokens is not None:  # smaller case (profiling)
        lens = inputs.multinomial_lens(args.groups or cfg["G"], args.tokens or cfg["M_total"],
                                       args.seed)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).to(device)
    M = int(lens.sum())
    g = torch.Generator(device=device).manual_seed(args.seed)
    x = torch.randn(M, cfg["OUT_M"], generator=g, device=device).to(torch.bfloat16)
    dy = torch.randn(M, cfg["OUT_N"], generator=g, device=device).to(torch.bfloat16)
    q_x = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=device)
    q_dy = torch.empty(dy.shape, dtype=torch.float8_e5m2, device=device)
    s_x = torch.empty(len(lens), dtype=torch.float32, device=device)
    s_dy = torch.empty_like(s_x)
    stream = torch.cuda.current_stream(device)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    per_kernel = {"x_e4m3": 0.0, "dy_e5m2": 0.0}

    def step(timed=False):
        if timed:
            evs[0].record(stream)
        quantize_fp8(x, offs, "e4m3", out=q_x, scales=s_x)
        if timed:
            evs[1].record(stream)
        quantize_fp8(dy, offs, "e5m2", out=q_dy, scales=s_dy)
        if timed:
            evs[2].record(stream)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during warm-up")
    sampler = ClockSampler(local)
    sampler.__enter__()
    time.sleep(0.05)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    clocks = sampler.window(t0, t1)
    sampler.__exit__()
    ms = ev0.elapsed_time(ev1) / args.steps
    for _ in range(args.steps):  # per-kernel split, separate pass
        step(timed=True)
        torch.cuda.synchronize()
        per_kernel["x_e4m3"] += evs[0].elapsed_time(evs[1]) / args.steps
        per_kernel["dy_e5m2"] += evs[1].elapsed_time(evs[2]) / args.steps
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during the timed region")
    bytes_x, bytes_dy = 3 * x.numel(), 3 * dy.numel()
    value = (bytes_x + bytes_dy) / (ms * 1e-3) / 1e9
    _fp8, hbm, src = measured_peaks()
    ach_dy = bytes_dy / (per_kernel["dy_e5m2"] * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": ach_dy, "peak": hbm, "unit": "GB/s",
                "frac": ach_dy / hbm, "traffic": profile_traffic("quantize_dy_gate_up"),
                "peak_source": ("of measured: MEASURED_PEAKS.json hbm_gbs (copy, read + write)"
                                if src.startswith("of measured") else "of fallback: 6.65 TB/s"),
                "kernel": "vark_quant_tma_kernel<e5m2> (dy, F=5760)",
                "algorithmic_unit": "3 bytes per element (2 read, 1 written) per launch"}
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import vark_oracle as vo

        torch.set_num_threads(os.cpu_count() or 1)
        done, secs = 0, 0.0
        for e in range(len(lens)):
            lo, hi = int(offs[e]), int(offs[e + 1])
            xc = dy[lo:hi].cpu()
            t_s = time.perf_counter()
            vo.quantize_fp8_ref(xc, [0, hi - lo], "e5m2")
            secs += time.perf_counter() - t_s
            done += 3 * xc.numel()
            if secs > args.cpu_seconds:
                break
        cpu = {"value": done / secs / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"dy experts 0..{e} quantised by the torch CPU oracle; "
                                         f"{secs:.1f} s"}
    line = {
        "metric": "producer step (per-expert amax + fp8 quantisation of x and dy) GB/s",
        "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 -> fp8 (e4m3 / e5m2)",
        "data": "synthetic (seeded N(0,1) bf16 on the device)",
        "config": {"workload": "quantize_gate_up", "G": len(lens), "M_total": M,
                   "F_x": cfg["OUT_M"], "F_dy": cfg["OUT_N"], "granularity": "group",
                   "l2": "inputs (2.26 GB) >> 126 MB L2; no flush"},
        "per_kernel_ms": per_kernel, "e2e": None, "roofline": roofline, "cpu_baseline": cpu,
        "clocks": clocks, "gpu_launches": 2 * args.steps,
    }
    print(json.dumps(line), flush=True)


FWD_SITES = {  # reference harness bench.py:154-181: (A dtype, N, K); M_total 131072, E 32
    "gate_up_fwd": ("e4m3", 5760, 2880), "down_fwd": ("e4m3", 2880, 2880),
    "down_dgrad": ("e5m2", 2880, 2880), "gate_up_dgrad": ("e5m2", 2880, 5760),
}


def run_fwd(args):
    """Fixed-K grouped GEMM at one harness site on one GPU (reference generator's routing,
    bench.py:205-212; N(0,1) cast to fp8 and scales 0.1 as bench.py:221-223,257-258). Metric:
    TFLOPS = 2 * M_total * N * K / time. A per-expert cuBLAS loop (torch._scaled_mm) is timed
    beside it for context."""
    from ggemm_asm_b200 import _lib, grouped_gemm_fp8_tensorwise, inputs

    rank, world, local = dist_env()
    if world != 1:
        raise SystemExit("--op fwd runs on one GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    a_fmt, N, K = FWD_SITES[args.site]
    G, M = args.groups or 32, args.tokens or 131072
    lens = inputs.reference_exponential_lens(G, M, seed=42)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).to(device)
    g = torch.Generator(device=device).manual_seed(args.seed)
    a_dtype = torch.float8_e4m3fn if a_fmt == "e4m3" else torch.float8_e5m2
    a = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16).to(a_dtype)
    b = torch.randn(G, N, K, generator=g, device=device).to(torch.bfloat16).to(torch.float8_e4m3fn)
    sa = torch.tensor([0.1], device=device)
    sb = torch.tensor([0.1], device=device)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        grouped_gemm_fp8_tensorwise(a, b, sa, sb, offs, out=out)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during warm-up")
    sampler = ClockSampler(local)
    sampler.__enter__()
    time.sleep(0.05)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    clocks = sampler.window(t0, t1)
    sampler.__exit__()
    ms = ev0.elapsed_time(ev1) / args.steps
    flops = 2.0 * M * N * K
    value = flops / (ms * 1e-3) / 1e12
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during the timed region")
    cublas = None
    if not args.no_cublas:
        # cuBLAS per expert: torch._scaled_mm(a_g, b_g^T) needs row-major A and column-major B;
        # b[g] is [N, K] row-major, so b[g].t() is column-major [K, N] as required.
        o = offs.tolist()
        try:
            def cub():
                for e in range(G):
                    if o[e + 1] > o[e]:
                        torch._scaled_mm(a[o[e]:o[e + 1]], b[e].t(), scale_a=sa, scale_b=sb,
                                         out_dtype=torch.bfloat16)
            for _ in range(3):
                cub()
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(args.steps):
                cub()
            ev1.record(stream)
            torch.cuda.synchronize()
            cms = ev0.elapsed_time(ev1) / args.steps
            cublas = {"ms": cms, "tflops": flops / (cms * 1e-3) / 1e12,
                      "what": "torch._scaled_mm per expert (cuBLAS), same data"}
        except Exception as exc:  # e.g. an fp8 combination cuBLAS does not take
            cublas = {"unavailable": f"{type(exc).__name__}: {str(exc)[:120]}"}
    cpu = None
    if not args.no_cpu_baseline:
        # The CPU restatement (oracle, torch fp32 per expert) on a bounded sample of experts.
        from oracle import vark_oracle as vo

        torch.set_num_threads(os.cpu_count() or 1)
        o = offs.tolist()
        done, secs, e = 0.0, 0.0, 0
        sa_c, sb_c = sa.cpu(), sb.cpu()
        for e in range(G):
            lo, hi = o[e], o[e + 1]
            if hi == lo:
                continue
            ac = a[lo:hi].cpu()
            bc = b[e:e + 1].cpu()
            t_s = time.perf_counter()
            vo.grouped_fwd_f32(ac, bc, sa_c, sb_c, [0, hi - lo])
            secs += time.perf_counter() - t_s
            done += 2.0 * (hi - lo) * N * K
            if secs > args.cpu_seconds:
                break
        cpu = {"value": done / secs / 1e12, "unit": "TFLOPS", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"experts 0..{e} by the torch CPU oracle; {secs:.1f} s"}
    fp8_peak, _hbm, peak_src = measured_peaks()
    line = {
        "metric": f"{args.site} fixed-K grouped FP8 GEMM TFLOPS", "value": value, "unit": "TFLOPS",
        "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"fp8({a_fmt} x e4m3) -> fp32 acc -> bf16",
        "data": "synthetic (N(0,1) cast to fp8, scales 0.1; reference exponential routing)",
        "config": {"workload": args.site, "G": G, "M_total": M, "N": N, "K": K,
                   "l2": "operands >> 126 MB L2; no flush"},
        "roofline": {"bound": "tensor", "achieved": value, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": value / fp8_peak, "peak_source": peak_src,
                     "frac_of_nominal_4500": value / FP8_NOMINAL_TFLOPS,
                     "kernel": "vark_fwd2_kernel", "traffic": profile_traffic(args.site)},
        "cublas_per_expert": cublas, "clocks": clocks, "gpu_launches": args.steps, "e2e": None,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def run_layer(args):
    """One training step (forward + backward) of the FP8 MoE expert linear layer at the gate_up
    shape (x [131072, 2880], W [32, 2880, 5760], multinomial routing): quantise x and W, forward
    GEMM, quantise dy, data-gradient GEMM, weight-gradient GEMM. Metric: TFLOPS of the three
    GEMMs (3 * 2*M*K*N) over the whole step. A bf16 per-expert torch (cuBLAS) loop of the same
    three products is timed beside it for context."""
    from ggemm_asm_b200 import _lib, inputs
    from ggemm_asm_b200.moe import grouped_linear_fp8

    rank, world, local = dist_env()
    if world != 1:
        raise SystemExit("--op layer runs on one GPU")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    cfg = inputs.CONFIGS["gate_up"]
    G, M, K, N = cfg["G"], cfg["M_total"], cfg["OUT_M"], cfg["OUT_N"]
    lens = inputs.config_lens("gate_up", args.seed)
    offs = torch.from_numpy(inputs.offsets_from_lens(lens)).to(device)
    g = torch.Generator(device=device).manual_seed(args.seed)
    x = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(G, K, N, generator=g, device=device) * K ** -0.5).to(torch.bfloat16)
    w.requires_grad_(True)
    dy = torch.randn(M, N, generator=g, device=device).to(torch.bfloat16)
    stream = torch.cuda.current_stream(device)

    def step():
        x.grad = None
        w.grad = None
        y = grouped_linear_fp8(x, w, offs)
        y.backward(dy)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during warm-up")
    sampler = ClockSampler(local)
    sampler.__enter__()
    time.sleep(0.05)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.window(t0, time.perf_counter())
    sampler.__exit__()
    ms = ev0.elapsed_time(ev1) / args.steps
    flops = 3 * 2.0 * M * K * N
    value = flops / (ms * 1e-3) / 1e12
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during the timed region")
    bf16 = None
    if not args.no_cublas:
        o = offs.tolist()
        xs = x.detach()
        ws = w.detach()

        def ref_step():
            for e in range(G):
                if o[e + 1] > o[e]:
                    xe, de = xs[o[e]:o[e + 1]], dy[o[e]:o[e + 1]]
                    torch.matmul(xe, ws[e])
                    torch.matmul(de, ws[e].t())
                    torch.matmul(xe.t(), de)
        for _ in range(2):
            ref_step()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(max(2, args.steps // 4)):
            ref_step()
        ev1.record(stream)
        torch.cuda.synchronize()
        bms = ev0.elapsed_time(ev1) / max(2, args.steps // 4)
        bf16 = {"ms": bms, "tflops": flops / (bms * 1e-3) / 1e12,
                "what": "bf16 torch.matmul per expert (cuBLAS): forward, dx, dW; no quantisation"}
    fp8_peak, _hbm, peak_src = measured_peaks()
    print(json.dumps({
        "metric": "FP8 MoE linear layer training step (fwd + dx + dW) TFLOPS", "value": value,
        "unit": "TFLOPS", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8 (e4m3 x, W; e5m2 dy) -> fp32 acc -> bf16, per-expert amax scales",
        "data": "synthetic (seeded N(0,1) bf16 x, dy; W ~ N(0, 1/K))",
        "config": {"workload": "moe_linear_gate_up", "G": G, "M_total": M, "K": K, "N": N},
        "roofline": {"bound": "tensor", "achieved": value, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": value / fp8_peak, "peak_source": peak_src,
                     "note": "includes the three quantisation passes (HBM bound)"},
        "bf16_cublas_per_expert": bf16, "clocks": clocks, "e2e": None, "cpu_baseline": None,
    }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.op == "quantize":
        run_quantize(args)
        return
    if args.op == "fwd":
        run_fwd(args)
        return
    if args.op == "layer":
        run_layer(args)
        return
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
        pg = dist

    from ggemm_asm_b200 import _lib, variable_k_wgrad

    p, scaling = build_problem(args, rank, world, device)
    out = torch.empty(p.G, p.OUT_M, p.OUT_N, dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        variable_k_wgrad(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs, out=out)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during warm-up")

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    # ---- kernel-only timed region -------------------------------------------------------------
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    sampler.__enter__()
    time.sleep(0.05)
    barrier()
    t_begin = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    t_end = time.perf_counter()
    barrier()
    clocks = sampler.window(t_begin, t_end)
    ms_local = ev0.elapsed_time(ev1) / args.steps
    fp8_peak, _hbm, peak_src = measured_peaks()

    # ---- the other wgrad workloads, each timed like the headline (outside its timed region) --
    # N = 1: down_wgrad and the skewed-routing stress problem (BASELINE configs 2 and 3). Every
    # N: the GPT-OSS-120B-shaped problem (config 4: G = 128, M_total = 1048576) split into
    # contiguous expert ranges across the ranks (strong scaling; at N = 1 the whole problem).
    # Each starts after a short idle, like the headline, so that it is not timed in the power
    # state the previous workload left behind; its own clock window is recorded.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def time_steps(fn, steps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        time.sleep(0.5)
        barrier()
        t0 = time.perf_counter()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        barrier()
        return e0.elapsed_time(e1) / steps, sampler.window(t0, t1)

    other = {}
    if args.config == "gate_up" and not args.no_other:
        from ggemm_asm_b200 import inputs, launch_raw

        # The reference-facing 14-argument entry point on the same problem: no M_total, so its
        # loads are bounded by group_offs[G] on the device.
        def drop_in():
            launch_raw(p.lhs.data_ptr(), p.rhs.data_ptr(), out.data_ptr(),
                       p.lhs_scale.data_ptr(), p.rhs_scale.data_ptr(), p.group_offs.data_ptr(),
                       p.G, p.OUT_M, p.OUT_N, p.lhs.stride(0), p.rhs.stride(0), out.stride(0),
                       out.stride(1), out.stride(2), stream.cuda_stream)

        d_ms, d_clocks = time_steps(drop_in, args.steps)
        other["gate_up_wgrad_14arg"] = {
            "value": _sum_over_ranks(pg, p.flops, device) / (max_over_ranks(d_ms) * 1e-3) / 1e12
            if pg is not None else p.flops / (d_ms * 1e-3) / 1e12,
            "unit": "TFLOPS", "ms_per_step": d_ms, "steps": args.steps, "clocks": d_clocks,
            "api": "ggemm_vark_fp8_wgrad (the 14-argument drop-in, M_total not given)"}

        names = (["down", "skew"] if world == 1 else []) + ["shard120b"]
        for name in names:
            if name == "shard120b":
                q, _ = build_problem(argparse.Namespace(**{**vars(args), "config": name}), rank,
                                     world, device)
            else:
                q = inputs.make_problem(name, seed=args.seed, device=device)
            qo = torch.empty(q.G, q.OUT_M, q.OUT_N, dtype=torch.bfloat16, device=device)
            # The 120B split's steps are sized so that its timed region lasts about as long as
            # the headline's at every N (a rank's share is 1/N of the problem): a much longer
            # region at N = 1 would run into the power cap and flatter the scaling.
            q_steps = args.steps if name != "shard120b" else max(2, round(args.steps * world / 8))
            q_ms, q_clocks = time_steps(lambda: variable_k_wgrad(q.lhs, q.rhs, q.lhs_scale,
                                                                 q.rhs_scale, q.group_offs,
                                                                 out=qo), q_steps)
            if name == "shard120b":
                per_ms = _gather_over_ranks(pg, q_ms, device)
                per_tok = _gather_over_ranks(pg, float(q.lens.sum()), device)
                q_flops = 2.0 * sum(per_tok) * q.OUT_M * q.OUT_N
                t = max(per_ms)
                other["shard120b_strong"] = {
                    "value": q_flops / (t * 1e-3) / 1e12, "unit": "TFLOPS",
                    "per_gpu": q_flops / (t * 1e-3) / 1e12 / world, "ms_per_step": t,
                    "per_rank_ms": per_ms, "per_rank_tokens": [int(v) for v in per_tok],
                    "per_rank_tflops": [2.0 * k * q.OUT_M * q.OUT_N / (m * 1e-3) / 1e12
                                        for k, m in zip(per_tok, per_ms)],
                    "scaling": "strong", "steps": q_steps, "clocks": q_clocks,
                    "config": {"G": 128, "M_total": 1048576, "OUT_M": q.OUT_M,
                               "OUT_N": q.OUT_N, "split": "contiguous expert ranges"}}
            else:
                other[f"{name}_wgrad"] = {
                    "value": q.flops / (q_ms * 1e-3) / 1e12, "unit": "TFLOPS",
                    "ms_per_step": q_ms, "steps": args.steps, "clocks": q_clocks,
                    "frac": q.flops / (q_ms * 1e-3) / 1e12 / fp8_peak,
                    "config": {"G": q.G, "M_total": q.M_total, "OUT_M": q.OUT_M,
                               "OUT_N": q.OUT_N}}
            del q, qo
            torch.cuda.empty_cache()
        if _lib.read_status(clear=True) != 0:
            raise SystemExit("device status flags set in the other workloads")

    # Sustained clocks: the same work continued (untimed) for about half a second, with its own
    # events, so that the line also shows the rate once the power cap has settled the clock.
    t_s0 = time.perf_counter()
    n_sus = 0
    ev0.record(stream)
    while time.perf_counter() - t_s0 < 0.5:
        for _ in range(10):
            step()
        n_sus += 10
        torch.cuda.synchronize()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks_sustained = sampler.window(t_s0 + 0.2, time.perf_counter())
    sampler.__exit__()
    sus_ms = ev0.elapsed_time(ev1) / n_sus
    sustained = {"value": p.flops / (sus_ms * 1e-3) / 1e12, "unit": "TFLOPS (this rank)",
                 "ms_per_step": sus_ms, "steps": n_sus, "sm_mhz": clocks_sustained.get("sm_mhz"),
                 "what": "the same call repeated for 0.5 s after the timed region, untimed"}
    ms = max_over_ranks(ms_local)
    flops_local = p.flops
    flops_total = flops_local if pg is None else _sum_over_ranks(pg, flops_local, device)
    value = flops_total / (ms * 1e-3) / 1e12
    if _lib.read_status(clear=True) != 0:
        raise SystemExit("device status flags set during the timed region")
    fp8_peak, _hbm, peak_src = measured_peaks()

    # ---- end-to-end: pinned host inputs -> device -> kernel -> result back to the host ------
    # Through the host-buffer entry point (HostWgrad): per step, the H2D copy of LHS, RHS, scales
    # and offsets from pinned host memory and the D2H copy of C, overlapped with the kernel in
    # expert chunks. The plain serial sequence (copy in, one call, copy out) is reported beside.
    e2e = None
    if not args.no_e2e:
        from ggemm_asm_b200.host import HostWgrad

        h_lhs = torch.empty(p.lhs.shape, dtype=p.lhs.dtype, pin_memory=True)
        h_rhs = torch.empty(p.rhs.shape, dtype=p.rhs.dtype, pin_memory=True)
        h_ls = torch.empty(p.lhs_scale.shape, dtype=torch.float32, pin_memory=True)
        h_rs = torch.empty(p.rhs_scale.shape, dtype=torch.float32, pin_memory=True)
        for h, d in ((h_lhs, p.lhs), (h_rhs, p.rhs), (h_ls, p.lhs_scale), (h_rs, p.rhs_scale)):
            h.copy_(d)
        h_offs_np = p.group_offs.cpu().numpy().copy()
        h_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        h2d = (sum(t.numel() * t.element_size() for t in (h_lhs, h_rhs, h_ls, h_rs))
               + h_offs_np.nbytes)
        d2h = h_out.numel() * h_out.element_size()
        pipe = HostWgrad(p.lhs.shape[0], p.G, p.OUT_M, p.OUT_N, device=device, chunks=16)

        def e2e_step():
            pipe(h_lhs, h_rhs, h_ls, h_rs, h_offs_np, h_out)

        e2e_step()
        torch.cuda.synchronize()
        e2e_steps = max(2, min(args.steps, 5))
        barrier()
        ev0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / e2e_steps)
        if not torch.equal(h_out.to(device), out):
            raise SystemExit("e2e output mismatch")

        # Serial reference sequence: copy everything in, one call, copy C out.
        d_lhs, d_rhs = torch.empty_like(p.lhs), torch.empty_like(p.rhs)
        d_ls, d_rs = torch.empty_like(p.lhs_scale), torch.empty_like(p.rhs_scale)
        d_offs = torch.empty_like(p.group_offs)
        h_offs = torch.from_numpy(h_offs_np).pin_memory()

        def serial_step():
            d_lhs.copy_(h_lhs, non_blocking=True)
            d_rhs.copy_(h_rhs, non_blocking=True)
            d_ls.copy_(h_ls, non_blocking=True)
            d_rs.copy_(h_rs, non_blocking=True)
            d_offs.copy_(h_offs, non_blocking=True)
            variable_k_wgrad(d_lhs, d_rhs, d_ls, d_rs, d_offs, out=out)
            h_out.copy_(out, non_blocking=True)

        serial_step()
        torch.cuda.synchronize()
        barrier()
        ev0.record(stream)
        for _ in range(e2e_steps):
            serial_step()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        serial_ms = max_over_ranks(ev0.elapsed_time(ev1) / e2e_steps)
        e2e = {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "steps": e2e_steps,
               "api": "ggemm_asm_b200.host.HostWgrad (16 expert chunks, copies overlapped)",
               "serial": {"value": flops_total / (serial_ms * 1e-3) / 1e12,
                          "ms_per_step": serial_ms,
                          "api": "copy in, one grouped_gemm_fp8_tensorwise_variable_k, copy out"}}

    # ---- roofline of the dominant kernel ------------------------------------------------------
    achieved = flops_local / (ms_local * 1e-3) / 1e12
    workload = f"{args.config}"
    roofline = {"bound": "tensor", "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                "frac": achieved / fp8_peak, "traffic": profile_traffic(workload),
                "peak_source": peak_src, "frac_of_nominal_4500": achieved / FP8_NOMINAL_TFLOPS,
                "kernel": "vark_tc2_kernel",
                "algorithmic_unit": "2*tokens*OUT_M*OUT_N FLOP per launch (this rank)"}

    # ---- CPU baseline (rank 0, N=1 only) --------------------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from ggemm_asm_b200 import inputs

        torch.set_num_threads(os.cpu_count() or 1)
        pc = inputs.Problem(**{**p.__dict__}).to("cpu")
        rate, sample, secs = cpu_oracle_rate(pc, args.cpu_seconds)
        cpu = {"value": rate, "unit": "TFLOPS", "cores": torch.get_num_threads(), "kind": "port",
               "sample": sample + f"; {secs:.1f} s", "os_cpu_count": os.cpu_count(),
               "same_as": "bench.py --impl reference (same sample steps)"}

    if rank == 0:
        line = {
            "metric": metric_name(args.config),
            "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": (value / world) / REF_PUBLISHED_TFLOPS if args.config == "gate_up" else None,
            "vs_baseline_note": "per-GPU value / 1237 TFLOPS (reference's best published gate_up "
                                "number: MI355X hand-optimised ASM, README.md:60)",
            "dtype": "fp8(e4m3 x e5m2) -> fp32 acc -> bf16",
            "data": "synthetic (seeded N(0,1), amax-scaled fp8)",
            "config": {"workload": f"{args.config}_wgrad", "G": p.G, "M_total": p.M_total,
                       "OUT_M": p.OUT_M, "OUT_N": p.OUT_N, "per_rank": True,
                       "parallelism": f"expert-shard x{world}",
                       "l2": "inputs (1.13 GB) >> 126 MB L2; no flush"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu,
            "clocks": clocks, "clocks_sustained_untimed": clocks_sustained,
            "sustained_untimed": sustained,
            "gpu_launches": args.steps,
            "gpu_launches_e2e": None if e2e is None else e2e["steps"],
            "other_workloads": other,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def _gather_over_ranks(pg, x: float, device) -> list[float]:
    """x from every rank, in rank order (outside any timed region)."""
    if pg is None:
        return [x]
    t = torch.tensor([x], dtype=torch.float64, device=device)
    out = torch.empty(pg.get_world_size(), dtype=torch.float64, device=device)
    pg.all_gather_into_tensor(out, t)
    return [float(v) for v in out.tolist()]


def _sum_over_ranks(pg, x: float, device) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return float(t.item())


if __name__ == "__main__":
    main()
