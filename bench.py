#!/usr/bin/env python3
"""Benchmark of the attention hot path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload train|decode|cp]

Default workload ("train") is BASELINE config 3: bf16 causal attention
forward + backward, global B=8 H=32 N=4096 D=128, synthetic inputs
(0.5*N(0,1) for Q/K/V, N(0,1) for dO).  One step = one forward and one
backward through the library's C ABI.  With N GPUs (torchrun, one process
per GPU) the 256 (batch, head) units of the global batch are split 256/N per
GPU ("strong" scaling; the [B,H,N,D] layout is [1, B*H, N, D], so a rank's
units are one contiguous slice); there is no collective on the data path.
The same line carries, measured in the same run:
  weak     (N > 1) every rank runs the whole B8 H32 problem;
  e2e      the step through the public API with host buffers (PCIe copies);
  cp       BASELINE config 5 (bf16 causal forward, B1 H32 N131072 D128)
           through the context-parallel ring entry over all N GPUs;
  decode   BASELINE config 4 (split-KV decode, num_splits swept) (N = 1);
  fp32     BASELINE config 1 forward and backward (N = 1);
  config2  BASELINE config 2 fp16 forward + backward (N = 1);
  cpu_baseline  the reference's CPU loops on a bounded sample (N = 1).

`--impl reference` times the reference's CPU implementation of the same step
(the restated CPU path in oracle/, all host threads, bounded row sample of
the same workload); under torchrun only rank 0 runs it.  Where a GPU and the
reference library built from its own sources (oracle/_ref) are present, its
line also carries that library's GPU time at config 3 (`reference_gpu`).
"""

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "cuflash-attn_b200"))

METRIC = "attn fwd & fwd+bwd TFLOP/s per GPU (% BF16 peak); split-KV decode HBM GB/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

TRAIN = dict(B=8, H=32, N=4096, D=128, causal=True)
DECODE = dict(B=64, H=32, N=16384, D=128)
CONFIG1 = dict(B=2, H=8, N=1024, D=64, causal=True)
CONFIG2 = dict(B=4, H=16, N=2048, D=128, causal=False)
CONFIG5 = dict(B=1, H=32, N=131072, D=128)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def tensor_peak(pk, pk_kind, clocks):
    """The dense bf16 peak of the regime the timed region ran in: the burst
    figure when the SM clock stayed at its maximum with no power capping,
    the sustained (power-capped) figure otherwise."""
    mhz, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    capped = "sw_power_cap" in (clocks.get("reasons") or [])
    burst = mhz is not None and mx and mhz >= 0.97 * mx and not capped
    key = "bf16_tflops" if burst else "bf16_tflops_sustained"
    return pk.get(key, FALLBACK_PEAKS[key]), f"{key} ({pk_kind})"


def fwd_flops(B, H, N, D, causal):
    f = 4.0 * B * H * N * N * D
    return f * 0.5 if causal else f


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Clocks:
    """Samples SM clock, power and clock-event reasons of one GPU every 10 ms
    during the timed region, through NVML (read-only queries) in a background
    thread; without NVML the summary says so instead of reporting clocks."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device_index):
        self.idx = device_index
        self.rows = []
        self.err = None
        self.thread = None

    def _handle(self, nv):
        try:
            import torch

            prop = torch.cuda.get_device_properties(self.idx)
            bus = "%08X:%02X:%02X.0" % (prop.pci_domain_id, prop.pci_bus_id, prop.pci_device_id)
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.idx)

    def __enter__(self):
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            masks = [(name, getattr(nv, const, 0)) for name, const in self.REASONS]
        except Exception as e:  # no NVML: report that instead of clocks
            self.err = f"nvml unavailable: {type(e).__name__}"
            return self
        self.stop = threading.Event()

        def run():
            while not self.stop.is_set():
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    mw = nv.nvmlDeviceGetPowerUsage(h)
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.rows.append((mhz, mw / 1000.0, [n for n, m in masks if m and bits & m]))
                except Exception as e:
                    self.err = f"nvml query failed: {type(e).__name__}"
                    return
                self.stop.wait(0.01)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.rows and self.err is None and time.time() - t0 < 2.0:
            time.sleep(0.002)
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0,
                    "reasons": [self.err or "no samples"]}
        reasons = sorted({r for row in self.rows for r in row[2]})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(r[0] for r in self.rows),
                "power_w_max": max(r[1] for r in self.rows), "samples": len(self.rows),
                "reasons": reasons}


def traffic_from_profiles(kernel_tag):
    """Per-launch DRAM bytes of `kernel_tag` from an ncu capture, summarised
    in profiles/dram_traffic.json (null when no capture has been summarised)."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel_tag, {}).get("bytes_per_launch")
    except (ValueError, AttributeError):
        return None


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def event_time(fn, steps, warmup, stream):
    """Mean ms per call of fn() over `steps` calls after `warmup`, CUDA events
    on `stream`."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def max_over_ranks(vals, dev, world):
    if world == 1:
        return vals
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


# ---------------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------------

def cpu_reference_step(Qh, Kh, Vh, dOh, scale, causal, threads, row_step):
    """One bounded sample of the reference CPU step; returns (algorithmic FLOPs, s)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    t0 = time.perf_counter()
    pairs = oracle.train_step_rows_f32(Qh, Kh, Vh, dOh, scale, causal, (0, threads), 0, row_step,
                                       threads)
    dt = time.perf_counter() - t0
    D = Qh.shape[2]
    return 3.5 * 4.0 * D * pairs, dt


def cpu_sample_inputs(threads, N, D):
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    shape = (threads, N, D)
    return (oracle.normal(shape, 21, 0.5), oracle.normal(shape, 22, 0.5),
            oracle.normal(shape, 23, 0.5), oracle.normal(shape, 24, 1.0))


def reference_gpu_times():
    """GPU time of the reference library (compiled from its own sources into
    oracle/_ref) at config 3 through its C ABI: one forward and one backward
    after a warm-up forward, CUDA events.  None without a GPU or that build."""
    try:
        import torch
    except ImportError:
        return None
    sys.path.insert(0, str(ROOT / "oracle"))
    import cuflash_attn
    import oracle

    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    if not oracle.REF_LIB_PATH.exists():
        return {"unavailable": "oracle/_ref/libcuflash_attn_ref.so not built"}
    ref = cuflash_attn.CuFlashAttn(str(oracle.REF_LIB_PATH), reference_abi_only=True)
    c = TRAIN
    B, H, N, D = c["B"], c["H"], c["N"], c["D"]
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(21)
    shape = (B, H, N, D)
    Q, K, V = ((0.5 * torch.randn(shape, device=dev, generator=g)).to(torch.bfloat16)
               for _ in range(3))
    dO = torch.randn(shape, device=dev, generator=g).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream()
    O, L = ref.forward(Q, K, V, causal=True, scale=scale)
    fwd_ms = event_time(lambda: ref.forward(Q, K, V, causal=True, scale=scale, O=O, L=L), 1, 1,
                        stream)
    bwd_ms = event_time(lambda: ref.backward(Q, K, V, O, L, dO, causal=True, scale=scale), 1, 0,
                        stream)
    ff = fwd_flops(B, H, N, D, True)
    return {"config": "BASELINE config 3 bf16 causal B8 H32 N4096 D128 (reference .so, sm_100a)",
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
            "fwd_tflops": ff / (fwd_ms * 1e-3) / 1e12,
            "fwd_bwd_tflops": 3.5 * ff / ((fwd_ms + bwd_ms) * 1e-3) / 1e12,
            "timing": "CUDA events, one call each after a warm-up forward"}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    c = TRAIN
    threads = min(host_threads(), 64)
    scale = 1.0 / math.sqrt(c["D"])
    Qh, Kh, Vh, dOh = cpu_sample_inputs(threads, c["N"], c["D"])
    row_step = 16  # 256 sampled rows per unit per step (about 1 s on one core)
    for _ in range(args.warmup):
        cpu_reference_step(Qh, Kh, Vh, dOh, scale, True, threads, row_step)
    flops = secs = 0.0
    for _ in range(args.steps):
        f, s = cpu_reference_step(Qh, Kh, Vh, dOh, scale, True, threads, row_step)
        flops += f
        secs += s
    tflops = flops / secs / 1e12
    sample = (f"{threads} (b,h) units of B8 H32 N4096 D128 causal, every {row_step}th query row, "
              "fp32 reference CPU loops (fwd+bwd rows)")
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3 bf16 causal fwd+bwd B8 H32 N4096 D128 (CPU sample)",
                   "global_batch": 8, "seq_len": 4096, "parallelism": "none"},
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if not args.skip_reference_gpu:
        try:
            line["reference_gpu"] = reference_gpu_times()
        except Exception as e:  # reported, never fatal for the CPU arm
            line["reference_gpu"] = {"unavailable": f"{type(e).__name__}: {e}"}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------

def make_train_inputs(dev, units, N, D, first_unit):
    """Config 3 inputs for (batch, head) units [first_unit, first_unit+units)
    of the global batch, as [1, units, N, D] (seeded per unit, so a unit's
    data does not depend on how the units are split over ranks)."""
    import torch

    shape = (1, units, N, D)
    Q, K, V, dO = (torch.empty(shape, device=dev, dtype=torch.bfloat16) for _ in range(4))
    for u in range(units):
        g = torch.Generator(device=dev).manual_seed(21 + 7919 * (first_unit + u))
        for t, std in ((Q, 0.5), (K, 0.5), (V, 0.5), (dO, 1.0)):
            t[0, u] = (std * torch.randn((N, D), device=dev, generator=g)).to(torch.bfloat16)
    return Q, K, V, dO


def time_train(lib, Q, K, V, dO, steps, warmup, stream, scale, clocks_dev=None):
    """Times `steps` forward+backward steps; returns ({total, fwd, bwd, bwd_main}
    ms, clocks summary, outputs)."""
    import torch

    O = torch.empty_like(Q)
    L = torch.empty(Q.shape[:3], device=Q.device, dtype=torch.float32)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        lib.forward(Q, K, V, causal=True, scale=scale, O=O, L=L, stream=stream)
        if ev is not None:
            ev[1].record(stream)
        lib.backward(Q, K, V, O, L, dO, causal=True, scale=scale, dQ=dQ, dK=dK, dV=dV,
                     stream=stream)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if lib.device_status() != 0:
        raise RuntimeError("kernel reported a wait timeout during warm-up")
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    barrier()
    torch.cuda.synchronize()
    clk = Clocks(clocks_dev) if clocks_dev is not None else None
    if clk is not None:
        clk.__enter__()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the library records an event pair around each backward main kernel
    # launch on this stream, so that kernel is timed apart from the
    # backward's preprocess and dQ-convert launches
    lib.profile_main_kernels(steps)
    t_start.record(stream)
    for k in range(steps):
        step(evs[k])
    t_end.record(stream)
    torch.cuda.synchronize()
    if clk is not None:
        clk.__exit__(None, None, None)
    barrier()
    main = lib.profile_read_ms(steps)
    lib.profile_main_kernels(0)
    if len(main) != steps:
        raise RuntimeError(f"{len(main)} backward main kernels profiled, expected {steps}")
    total = t_start.elapsed_time(t_end)
    fwd = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
    bwd = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
    times = {"total": total, "fwd": fwd, "bwd": bwd, "bwd_main": sum(main) / steps}
    return times, (clk.summary() if clk is not None else None), (O, L, dQ, dK, dV)


def barrier():
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def run_ours(args):
    import torch
    import torch.distributed as dist

    import cuflash_attn

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    lib = cuflash_attn.CuFlashAttn()
    stream = torch.cuda.current_stream()
    pk, pk_kind = peaks()

    if args.workload == "decode":
        line = run_decode(args, lib, dev, pk, pk_kind)
        if rank == 0:
            print(json.dumps(line), flush=True)
        return finish(world)
    if args.workload == "cp":
        line = run_cp(args, dev, world, rank, pk, pk_kind, backward=args.cp_backward,
                      steps=args.steps, warmup=args.warmup)
        if rank == 0:
            print(json.dumps(line), flush=True)
        return finish(world)

    # ---- config 3, (batch, head) units split over the ranks -----------------------
    N, D = args.seq, args.head_dim
    total_units = args.batch * args.heads
    base, extra = divmod(total_units, world)
    units = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    scale = 1.0 / math.sqrt(D)
    Q, K, V, dO = make_train_inputs(dev, units, N, D, first)
    warmup = max(args.warmup, 3)
    times, clocks, outs = time_train(lib, Q, K, V, dO, args.steps, warmup, stream, scale,
                                     clocks_dev=local)
    total_ms, fwd_ms, bwd_ms, main_ms = max_over_ranks(
        [times["total"], times["fwd"], times["bwd"], times["bwd_main"]], dev, world)
    ff_global = fwd_flops(1, total_units, N, D, True)
    step_flops = 3.5 * ff_global  # forward + backward (backward = 2.5 x forward)
    ms_step = total_ms / args.steps
    value = step_flops / (ms_step * 1e-3) / 1e12
    # per-kernel-family roofline of this rank's share (the slowest rank's times)
    ff_rank = fwd_flops(1, units if world == 1 else base + (1 if extra else 0), N, D, True)
    fwd_tflops = ff_rank / (fwd_ms * 1e-3) / 1e12
    bwd_tflops = 2.5 * ff_rank / (bwd_ms * 1e-3) / 1e12
    main_tflops = 2.5 * ff_rank / (main_ms * 1e-3) / 1e12
    peak, peak_src = tensor_peak(pk, pk_kind, clocks)
    # the dominant kernel: the backward's main kernel (timed by the library's
    # event pair around its launch) or the forward kernel (the only launch of
    # a forward call)
    dominant = "bwd" if main_ms >= fwd_ms else "fwd"
    achieved = main_tflops if dominant == "bwd" else fwd_tflops
    launches_per_step = 1 + lib_bwd_launches()

    # ---- end to end through the public API with host buffers --------------------
    e2e_ms, h2d, d2h = run_e2e(lib, Q, K, V, dO, outs, stream, dev, args.steps, scale)
    e2e_ms = max_over_ranks([e2e_ms], dev, world)[0]
    del outs

    # ---- weak scaling (N > 1): every rank runs the whole B8 H32 problem ---------
    weak = None
    if world > 1 and not args.skip_extras:
        del Q, K, V, dO
        torch.cuda.empty_cache()
        Qw, Kw, Vw, dOw = make_train_inputs(dev, total_units, N, D, 0)
        wsteps = min(args.steps, 10)
        w_times, _, o = time_train(lib, Qw, Kw, Vw, dOw, wsteps, 3, stream, scale)
        del o, Qw, Kw, Vw, dOw
        w_ms = max_over_ranks([w_times["total"] / wsteps], dev, world)[0]
        weak = {"value": world * step_flops / (w_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "ms_per_step": w_ms, "steps": wsteps,
                "workload": f"whole B{args.batch} H{args.heads} problem on every GPU"}
    else:
        del Q, K, V, dO
    torch.cuda.empty_cache()

    # ---- config 5 through the context-parallel ring over all ranks -------------
    cp = cp_train = None
    if not args.skip_extras:
        cp = run_cp(args, dev, world, rank, pk, pk_kind, backward=False,
                    steps=min(args.steps, 5 if world == 1 else 10), warmup=2)
        torch.cuda.empty_cache()
        # the training step of config 5: ring forward + ring backward
        cp_train = run_cp(args, dev, world, rank, pk, pk_kind, backward=True,
                          steps=min(args.steps, 3 if world == 1 else 5), warmup=1)
        torch.cuda.empty_cache()

    # ---- single-GPU extras (N = 1) ----------------------------------------------
    decode = fp32 = config2 = None
    if world == 1 and not args.skip_extras:
        decode = run_decode(args, lib, dev, pk, pk_kind, steps=min(args.steps, 10))
        torch.cuda.empty_cache()
        fp32 = run_fp32(lib, dev, stream, min(args.steps, 20), pk)
        config2 = run_config2(lib, dev, stream, min(args.steps, 20), pk, pk_kind)
        torch.cuda.empty_cache()

    # ---- CPU baseline (rank 0, N = 1 only) ---------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu_baseline:
        threads = min(host_threads(), 64)
        Qh, Kh, Vh, dOh = cpu_sample_inputs(threads, N, D)
        row_step = 8
        f, s = cpu_reference_step(Qh, Kh, Vh, dOh, scale, True, threads, row_step)
        cpu = {"value": f / s / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{threads} (b,h) units x every {row_step}th query row of B8 H32 N4096 "
                         f"D128 causal fwd+bwd, fp32 reference CPU loops, {s:.1f} s"}

    if rank == 0:
        traffic = traffic_from_profiles("bwd" if dominant == "bwd" else "fwd")
        is_c3 = (args.batch, args.heads, N, D) == (8, 32, 4096, 128)
        burst = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        sustained = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (torch.randn per (batch, head) unit, seed 21 + 7919*unit; "
                    "Q/K/V 0.5*N(0,1), dO N(0,1))",
            "config": {"workload": ("BASELINE config 3: " if is_c3 else "custom shape: ") +
                                   f"bf16 causal attention fwd+bwd, B{args.batch} H{args.heads} "
                                   f"N{N} D{D} (global)",
                       "global_batch": args.batch, "heads": args.heads, "seq_len": N,
                       "head_dim": D, "units_per_gpu": units if world == 1 else
                       f"{base}{'+1' if extra else ''}",
                       "parallelism": f"(batch,head) split {total_units}/{world} over "
                                      f"{world} GPU(s), no collective",
                       "l2": f"inputs ({4 * units * N * D * 2 / 2**20:.0f} MiB per GPU) vs "
                             "126 MB L2; no flush"},
            "value_is": "whole-job TFLOP/s over n_gpus (the metric's per-GPU figure: "
                        "per_gpu_tflops)",
            "per_gpu_tflops": value / world,
            "fwd": {"ms": fwd_ms, "tflops": fwd_tflops, "frac_burst": fwd_tflops / burst,
                    "frac_sustained": fwd_tflops / sustained},
            "bwd": {"ms": bwd_ms, "tflops": bwd_tflops, "frac_burst": bwd_tflops / burst,
                    "frac_sustained": bwd_tflops / sustained,
                    "main_kernel_ms": main_ms, "main_kernel_tflops": main_tflops,
                    "aux_kernels_ms": bwd_ms - main_ms},
            "roofline": {"bound": "tensor",
                         "kernel": "fa_bwd_kernel<bf16,128> (backward main kernel)"
                                   if dominant == "bwd" else "fa_fwd_kernel<bf16,128,0>",
                         "timed": "CUDA events recorded by the library around each launch of "
                                  "that kernel on the bench stream, averaged over the timed steps"
                                  if dominant == "bwd" else
                                  "CUDA events around each forward call (one launch)",
                         "algorithmic_flops_per_launch": (2.5 if dominant == "bwd" else 1.0)
                                                          * ff_rank,
                         "achieved": achieved,
                         "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": peak_src, "frac_burst": achieved / burst,
                         "frac_sustained": achieved / sustained, "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                           "per launch (profiles/dram_traffic.json)"},
            "cpu_baseline": cpu,
            "e2e": {"value": step_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "weak": weak,
            "cp": cp,
            "cp_train": cp_train,
            "decode": decode,
            "fp32": fp32,
            "config2": config2,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    return finish(world)


def finish(world):
    import torch.distributed as dist

    if world > 1 and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


def lib_bwd_launches():
    """Kernels one backward call launches (preprocess + main + dQ convert)."""
    return 3


def run_e2e(lib, Q, K, V, dO, outs, stream, dev, steps, scale):
    """The step through the public API with host buffers.  Every step copies
    its inputs Q, K, V, dO from pinned host memory and its outputs O, L, dQ,
    dK, dV back.  As in a training input pipeline, step k+1's inputs travel
    host->device while step k computes and step k-1's outputs travel
    device->host (PCIe is full duplex): three streams, device tensors
    double-buffered, ordered with events.  Returns (ms per step, h2d, d2h
    bytes per step)."""
    import torch

    O, L, dQ, dK, dV = outs
    e2e_steps = max(10, min(steps, 20))
    hQ, hK, hV, hdO = (x.cpu().pin_memory() for x in (Q, K, V, dO))
    hO = torch.empty_like(hQ, device="cpu").pin_memory()
    hL = torch.empty(L.shape, dtype=L.dtype).pin_memory()
    hdQ, hdK, hdV = (torch.empty_like(hQ, device="cpu").pin_memory() for _ in range(3))
    bufs = [dict(Q=Q, K=K, V=V, dO=dO, O=O, L=L, dQ=dQ, dK=dK, dV=dV)]
    bufs.append({k: torch.empty_like(v) for k, v in bufs[0].items()})
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    n_ev = e2e_steps + 2
    state = {}

    def new_events():
        state["in"] = [torch.cuda.Event() for _ in range(n_ev)]    # inputs of step k on device
        state["comp"] = [torch.cuda.Event() for _ in range(n_ev)]  # step k computed
        state["out"] = [torch.cuda.Event() for _ in range(n_ev)]   # step k's outputs on host

    def e2e_step(k):
        b = bufs[k % 2]
        ev_in, ev_comp, ev_out = state["in"], state["comp"], state["out"]
        with torch.cuda.stream(s_h2d):
            if k >= 2:
                s_h2d.wait_event(ev_comp[k - 2])  # step k-2 is done with these inputs
            for name, h in (("Q", hQ), ("K", hK), ("V", hV), ("dO", hdO)):
                b[name].copy_(h, non_blocking=True)
            ev_in[k].record(s_h2d)
        stream.wait_event(ev_in[k])
        if k >= 2:
            stream.wait_event(ev_out[k - 2])  # step k-2's outputs have left these buffers
        lib.forward(b["Q"], b["K"], b["V"], causal=True, scale=scale, O=b["O"], L=b["L"],
                    stream=stream)
        lib.backward(b["Q"], b["K"], b["V"], b["O"], b["L"], b["dO"], causal=True, scale=scale,
                     dQ=b["dQ"], dK=b["dK"], dV=b["dV"], stream=stream)
        ev_comp[k].record(stream)
        with torch.cuda.stream(s_d2h):
            s_d2h.wait_event(ev_comp[k])
            for name, h in (("O", hO), ("L", hL), ("dQ", hdQ), ("dK", hdK), ("dV", hdV)):
                h.copy_(b[name], non_blocking=True)
            ev_out[k].record(s_d2h)

    new_events()
    for k in range(2):  # warm the pipeline's streams and buffers
        e2e_step(k)
    torch.cuda.synchronize()
    new_events()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_h2d.wait_event(e0)
    for k in range(e2e_steps):
        e2e_step(k)
    stream.wait_stream(s_d2h)
    stream.wait_stream(s_h2d)
    e1.record(stream)
    torch.cuda.synchronize()
    h2d = 4 * Q.numel() * Q.element_size()
    d2h = 4 * Q.numel() * Q.element_size() + L.numel() * 4
    return e0.elapsed_time(e1) / e2e_steps, h2d, d2h


def run_decode(args, lib, dev, pk, pk_kind, steps=None):
    """BASELINE config 4 (or --kv-heads grouped-query): every num_splits of
    the sweep, CUDA events; returns the line / sub-object."""
    import torch

    c = DECODE
    steps = steps or args.steps
    B = args.batch if (args.workload == "decode" and args.batch_set) else c["B"]
    H, N = c["H"], c["N"]
    D = args.head_dim if args.workload == "decode" else c["D"]
    Hkv = (args.kv_heads or H) if args.workload == "decode" else H
    is_config4 = B == c["B"] and Hkv == H and D == c["D"]
    g = torch.Generator(device=dev).manual_seed(31)
    q = torch.randn((B, H, 1, D), device=dev, generator=g).to(torch.bfloat16)
    K = torch.randn((B, Hkv, N, D), device=dev, generator=g).to(torch.bfloat16)
    V = torch.randn((B, Hkv, N, D), device=dev, generator=g).to(torch.bfloat16)
    O = torch.empty_like(q)
    L = torch.empty((B, H), device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream()
    nbytes = 2 * B * Hkv * N * D * 2 + 2 * B * H * D * 2 + B * H * 4
    call = lib.decode if Hkv == H else lib.decode_gqa
    ps = args.page_size if args.workload == "decode" else 0
    if ps:
        # the same cache as pages [B*N/ps, ps, Hkv, D] in a shuffled order,
        # addressed through a block table (seeded permutation)
        npg = B * (N // ps)
        perm = torch.randperm(npg, device=dev, generator=g).to(torch.int32)
        table = perm.view(B, N // ps).contiguous()
        Kp = torch.empty((npg, ps, Hkv, D), device=dev, dtype=torch.bfloat16)
        Vp = torch.empty_like(Kp)
        Kp[perm.long()] = K.view(B, Hkv, N // ps, ps, D).permute(0, 2, 3, 1, 4).reshape(npg, ps, Hkv, D)
        Vp[perm.long()] = V.view(B, Hkv, N // ps, ps, D).permute(0, 2, 3, 1, 4).reshape(npg, ps, Hkv, D)
        lens = torch.full((B,), N, device=dev, dtype=torch.int32)
        del K, V
        K, V = Kp, Vp

        def call(q_, K_, V_, num_splits, O, L, stream):
            return lib.decode_paged(q_, K_, V_, table, lens, num_splits=num_splits, O=O, L=L,
                                    stream=stream)
    results = {}
    with Clocks(dev.index) as clk:
        for splits in args.splits:
            ms = event_time(lambda: call(q, K, V, num_splits=splits, O=O, L=L, stream=stream),
                            steps, 3, stream)
            results[splits] = {"ms": ms, "GBps": nbytes / (ms * 1e-3) / 1e9}
    del q, K, V
    best = max(results, key=lambda s: results[s]["GBps"])
    peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    return {
        "metric": METRIC, "value": results[best]["GBps"], "unit": "GB/s", "n_gpus": 1,
        "steps": steps, "warmup": 3, "ms_per_step": results[best]["ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (torch.randn, seed 31)",
        "config": {"workload": ("BASELINE config 4: " if is_config4 and not ps else "custom: ") +
                               (f"split-KV decode B{B} H{H} Nkv{N} D{D}" if Hkv == H else
                                f"grouped-query split-KV decode B{B} Hq{H} Hkv{Hkv} Nkv{N} D{D}") +
                               (f", paged cache ({ps}-row pages, shuffled block table)" if ps
                                else ""),
                   "best_num_splits": best, "bytes_per_call": nbytes,
                   "l2": f"K/V {2 * B * Hkv * N * D * 2 / 2**30:.1f} GiB vs 126 MB L2; no flush"},
        "splits": results,
        "roofline": {"bound": "hbm", "achieved": results[best]["GBps"], "peak": peak,
                     "unit": "GB/s", "frac": results[best]["GBps"] / peak,
                     "peak_source": f"hbm_gbs ({pk_kind})",
                     "traffic": traffic_from_profiles("decode") if is_config4 and not ps
                     else None},
        "clocks": clk.summary(),
    }


def run_fp32(lib, dev, stream, steps, pk):
    """BASELINE config 1 (fp32 causal, B2 H8 N1024 D64, U[-1,1]) forward and
    backward on the 3xTF32 tensor-core kernels."""
    import torch

    c = CONFIG1
    B, H, N, D = c["B"], c["H"], c["N"], c["D"]
    g = torch.Generator(device=dev).manual_seed(1)
    Q, K, V, dO = (torch.rand((B, H, N, D), device=dev, generator=g) * 2 - 1 for _ in range(4))
    scale = 1.0 / math.sqrt(D)
    O, L = lib.forward(Q, K, V, causal=True, scale=scale)
    f = event_time(lambda: lib.forward(Q, K, V, causal=True, scale=scale, O=O, L=L, stream=stream),
                   steps, 3, stream)
    b = event_time(lambda: lib.backward(Q, K, V, O, L, dO, causal=True, scale=scale,
                                        stream=stream), steps, 3, stream)
    ff = fwd_flops(B, H, N, D, True)
    tf32 = 1100.0  # nominal dense TF32 tensor peak of a B200 (no measured figure exists)
    return {"config": "BASELINE config 1: fp32 causal B2 H8 N1024 D64 (3xTF32 tcgen05)",
            "fwd_ms": f, "bwd_ms": b, "fwd_tflops": ff / (f * 1e-3) / 1e12,
            "bwd_tflops": 2.5 * ff / (b * 1e-3) / 1e12,
            "frac_of_3xtf32_nominal": {"fwd": ff / (f * 1e-3) / 1e12 / (tf32 / 3),
                                       "bwd": 2.5 * ff / (b * 1e-3) / 1e12 / (tf32 / 3)},
            "peak_note": "3xTF32 = 3 tf32 MMAs per product; nominal dense TF32 1.1 PFLOP/s"}


def run_config2(lib, dev, stream, steps, pk, pk_kind):
    """BASELINE config 2 (fp16 non-causal, B4 H16 N2048 D128) forward and
    backward."""
    import torch

    c = CONFIG2
    B, H, N, D = c["B"], c["H"], c["N"], c["D"]
    g = torch.Generator(device=dev).manual_seed(11)
    Q, K, V, dO = (torch.randn((B, H, N, D), device=dev, generator=g).to(torch.float16)
                   for _ in range(4))
    scale = 1.0 / math.sqrt(D)
    O, L = lib.forward(Q, K, V, causal=False, scale=scale)
    f = event_time(lambda: lib.forward(Q, K, V, causal=False, scale=scale, O=O, L=L,
                                       stream=stream), steps, 3, stream)
    b = event_time(lambda: lib.backward(Q, K, V, O, L, dO, causal=False, scale=scale,
                                        stream=stream), steps, 3, stream)
    ff = fwd_flops(B, H, N, D, False)
    burst = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    return {"config": "BASELINE config 2: fp16 non-causal B4 H16 N2048 D128",
            "fwd_ms": f, "bwd_ms": b, "fwd_tflops": ff / (f * 1e-3) / 1e12,
            "bwd_tflops": 2.5 * ff / (b * 1e-3) / 1e12,
            "fwd_bwd_tflops": 3.5 * ff / ((f + b) * 1e-3) / 1e12,
            "frac_burst": 3.5 * ff / ((f + b) * 1e-3) / 1e12 / burst,
            "peak_source": f"bf16_tflops ({pk_kind}; fp16 dense peak = bf16's)"}


def run_cp(args, dev, world, rank, pk, pk_kind, backward, steps, warmup):
    """causal forward (and, with `backward`, the ring
    backward of the training step) over B1 H32 N131072 D128, through the
    library's context-parallel ring entry (cuflash_attention_*_cp_bf16, NCCL
    send/recv of K/V between the zigzag shards of all ranks)."""
    import torch
    import torch.distributed as dist

    import ring_cp

    c = CONFIG5
    B, H, N, D = c["B"], c["H"], args.cp_seq, c["D"]
    C = N // (2 * world)
    scale = 1.0 / math.sqrt(D)
    chunks = ring_cp.zigzag_chunks(rank, world)

    def chunk_tensor(kind, ch):
        g = torch.Generator(device=dev).manual_seed(41 + 100 * kind + 7919 * ch)
        return torch.randn((B, H, C, D), device=dev, generator=g).to(torch.bfloat16)

    q_ab = [chunk_tensor(0, ch) for ch in chunks]
    k_ab = [chunk_tensor(1, ch) for ch in chunks]
    v_ab = [chunk_tensor(2, ch) for ch in chunks]
    do_ab = [chunk_tensor(3, ch) for ch in chunks] if backward else None
    comm = None
    if world > 1:
        uid = [ring_cp.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ring_cp.NcclComm(world, rank, uid[0])
    ring = ring_cp.RingAttention(comm, rank=rank, world=world, reserve_sms=args.cp_reserve)
    stream = torch.cuda.current_stream()

    def step():
        outs, lses = ring.forward(q_ab, k_ab, v_ab, scale)
        if backward:
            ring.backward(q_ab, k_ab, v_ab, outs, lses, do_ab, scale)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks([e0.elapsed_time(e1) / steps], dev, world)[0]
    barrier()
    if comm is not None:
        comm.destroy()
    flops = fwd_flops(B, H, N, D, True) * (3.5 if backward else 1.0)
    value = flops / (ms * 1e-3) / 1e12
    clocks = clk.summary()
    peak, peak_src = tensor_peak(pk, pk_kind, clocks)
    return {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (torch.randn per global chunk, seed 41+...)",
        "config": {"workload": f"BASELINE config 5: causal "
                               f"{'fwd+bwd' if backward else 'fwd'} B{B} H{H} N{N} D{D}, "
                               f"context-parallel ring over {world} GPU(s) "
                               f"(cuflash_attention_{'fwd+bwd' if backward else 'forward'}_cp_bf16,"
                               f" NCCL), zigzag chunks of {C}",
                   "global_batch": B, "seq_len": N, "parallelism": f"cp{world}",
                   "reserve_sms": args.cp_reserve},
        "per_gpu_tflops": value / world,
        "frac_per_gpu": value / world / peak, "peak_source": peak_src,
        "clocks": clocks,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["train", "decode", "cp"], default="train")
    ap.add_argument("--cp-seq", type=int, default=CONFIG5["N"])
    ap.add_argument("--cp-reserve", type=int, default=-1,
                    help="cp workload: SMs the step kernels leave to NCCL's transfer kernels "
                         "(-1 = the library's default)")
    ap.add_argument("--cp-backward", action="store_true",
                    help="cp workload: time the ring forward and backward of a training step")
    ap.add_argument("--splits", type=int, nargs="*", default=[0, 1, 2, 4, 8, 16, 32, 64])
    ap.add_argument("--kv-heads", type=int, default=0,
                    help="decode workload: K/V heads (fewer than the 32 query heads: grouped-query)")
    ap.add_argument("--page-size", type=int, default=0,
                    help="decode workload: read the cache through a paged layout with this many "
                         "rows per page (power of two; 0 = contiguous)")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-extras", action="store_true",
                    help="train workload: only config 3 (no weak/cp/decode/fp32/config2 fields)")
    ap.add_argument("--skip-reference-gpu", action="store_true")
    ap.add_argument("--batch", type=int, default=TRAIN["B"])
    ap.add_argument("--heads", type=int, default=TRAIN["H"])
    ap.add_argument("--seq", type=int, default=TRAIN["N"])
    ap.add_argument("--head-dim", type=int, default=TRAIN["D"])
    args = ap.parse_args()
    args.batch_set = any(a == "--batch" or a.startswith("--batch=") for a in sys.argv[1:])
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
