#!/usr/bin/env python3
"""Benchmark of the attention hot path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload train|decode]

Default workload ("train") is BASELINE config 3: bf16 causal attention
forward + backward, B=8 H=32 N=4096 D=128 per GPU, synthetic inputs
(0.5*N(0,1) for Q/K/V, N(0,1) for dO).  One step = one forward and one
backward through the library's C ABI.  Multi-GPU runs (torchrun, one process
per GPU) shard the global batch by (batch, head): every rank owns a fixed
B=8 x H=32 slice and there is no collective on the data path ("weak").

`--impl reference` times the reference's CPU implementation of the same step
(the restated CPU path in oracle/, all host threads, bounded row sample of
the same workload); under torchrun only rank 0 runs it.
"""

import argparse
import ctypes
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


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


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
    """Per-launch DRAM bytes of `kernel_tag` recorded from an ncu capture in
    profiles/dram_traffic.json (null when no capture has been summarised)."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel_tag, {}).get("bytes_per_launch")
    except (ValueError, AttributeError):
        return None


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


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
        "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3 bf16 causal fwd+bwd B8 H32 N4096 D128 (CPU sample)",
                   "global_batch": 8 * args.gpus, "seq_len": 4096, "parallelism": "none"},
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------

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
        return run_decode(args, lib, dev, world, rank, pk, pk_kind)
    if args.workload == "cp":
        return run_cp(args, lib, dev, world, rank, pk, pk_kind)

    B, H, N, D = args.batch, args.heads, args.seq, args.head_dim
    scale = 1.0 / math.sqrt(D)
    g = torch.Generator(device=dev).manual_seed(21 + 1000 * rank)
    shape = (B, H, N, D)
    Q = (0.5 * torch.randn(shape, device=dev, generator=g)).to(torch.bfloat16)
    K = (0.5 * torch.randn(shape, device=dev, generator=g)).to(torch.bfloat16)
    V = (0.5 * torch.randn(shape, device=dev, generator=g)).to(torch.bfloat16)
    dO = torch.randn(shape, device=dev, generator=g).to(torch.bfloat16)
    O = torch.empty_like(Q)
    L = torch.empty((B, H, N), device=dev, dtype=torch.float32)
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

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if lib.device_status() != 0:
        raise RuntimeError("kernel reported a wait timeout during warm-up")

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for k in range(args.steps):
            step(evs[k])
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    if world > 1:
        t = torch.tensor([total_ms, fwd_ms, bwd_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, fwd_ms, bwd_ms = (float(x) for x in t.tolist())

    ff = fwd_flops(B, H, N, D, True)
    step_flops = 3.5 * ff  # forward + backward (backward = 2.5 x forward)
    ms_step = total_ms / args.steps
    value = world * step_flops / (ms_step * 1e-3) / 1e12
    peak = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    fwd_tflops = ff / (fwd_ms * 1e-3) / 1e12
    bwd_tflops = 2.5 * ff / (bwd_ms * 1e-3) / 1e12
    dominant = "bwd" if bwd_ms >= fwd_ms else "fwd"
    achieved = bwd_tflops if dominant == "bwd" else fwd_tflops
    launches_per_step = 1 + lib_bwd_launches()

    # ---- end to end through the public API with host buffers --------------------
    # Every step copies its inputs Q, K, V, dO from pinned host memory and its
    # outputs O, L, dQ, dK, dV back, through the library's public calls.  As in
    # a training input pipeline, step k+1's inputs travel host->device while
    # step k computes and step k-1's outputs travel device->host (PCIe is full
    # duplex): three streams, device tensors double-buffered, ordered with
    # events.
    e2e_steps = max(10, min(args.steps, 20))
    hQ, hK, hV, hdO = (x.cpu().pin_memory() for x in (Q, K, V, dO))
    hO = torch.empty_like(hQ, device="cpu").pin_memory()
    hL = torch.empty(L.shape, dtype=L.dtype).pin_memory()
    hdQ, hdK, hdV = (torch.empty_like(hQ, device="cpu").pin_memory() for _ in range(3))
    bufs = [dict(Q=Q, K=K, V=V, dO=dO, O=O, L=L, dQ=dQ, dK=dK, dV=dV)]
    bufs.append({k: torch.empty_like(v) for k, v in bufs[0].items()})
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    n_ev = e2e_steps + 2
    ev_in = [torch.cuda.Event() for _ in range(n_ev)]     # inputs of step k on the device
    ev_comp = [torch.cuda.Event() for _ in range(n_ev)]   # step k computed
    ev_out = [torch.cuda.Event() for _ in range(n_ev)]    # step k's outputs on the host

    def e2e_step(k):
        b = bufs[k % 2]
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

    for k in range(2):  # warm the pipeline's streams and buffers
        e2e_step(k)
    torch.cuda.synchronize()
    ev_in = [torch.cuda.Event() for _ in range(n_ev)]
    ev_comp = [torch.cuda.Event() for _ in range(n_ev)]
    ev_out = [torch.cuda.Event() for _ in range(n_ev)]
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_h2d.wait_event(e0)
    for k in range(e2e_steps):
        e2e_step(k)
    stream.wait_stream(s_d2h)
    stream.wait_stream(s_h2d)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = 4 * Q.numel() * Q.element_size()
    d2h = 4 * Q.numel() * Q.element_size() + L.numel() * 4

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
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (torch.randn, seeds 21+1000*rank; Q/K/V 0.5*N(0,1), dO N(0,1))",
            "config": {"workload": ("BASELINE config 3: " if (B, H, N, D) == (8, 32, 4096, 128)
                                    else "custom shape: ") +
                                   f"bf16 causal attention fwd+bwd, B{B} H{H} N{N} D{D} per GPU",
                       "global_batch": B * world, "heads": 32, "seq_len": N, "head_dim": D,
                       "parallelism": f"(batch,head) sharding, {world} GPU(s), no collective",
                       "l2": f"inputs ({4 * Q.numel() * 2 / 2**20:.0f} MiB per GPU) vs 126 MB L2; "
                             "no flush"},
            "per_gpu_tflops": value / world,
            "pct_bf16_peak_per_gpu": 100.0 * (value / world) / peak,
            "fwd": {"ms": fwd_ms, "tflops": fwd_tflops,
                    "pct_peak": 100.0 * fwd_tflops / peak},
            "bwd": {"ms": bwd_ms, "tflops": bwd_tflops,
                    "pct_peak": 100.0 * bwd_tflops / peak},
            "roofline": {"bound": "tensor", "kernel": dominant, "achieved": achieved,
                         "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"bf16_tflops_sustained ({pk_kind})",
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": world * step_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def lib_bwd_launches():
    """Kernels one backward call launches (preprocess + main + dQ convert)."""
    return 3


def run_decode(args, lib, dev, world, rank, pk, pk_kind):
    import torch
    import torch.distributed as dist

    c = DECODE
    B, H, N, D = (args.batch if args.batch_set else c["B"]), c["H"], c["N"], args.head_dim
    Hkv = args.kv_heads or H  # fewer K/V heads than query heads: grouped-query decode
    is_config4 = B == c["B"] and Hkv == H and D == c["D"]
    g = torch.Generator(device=dev).manual_seed(31 + 1000 * rank)
    q = torch.randn((B, H, 1, D), device=dev, generator=g).to(torch.bfloat16)
    K = torch.randn((B, Hkv, N, D), device=dev, generator=g).to(torch.bfloat16)
    V = torch.randn((B, Hkv, N, D), device=dev, generator=g).to(torch.bfloat16)
    O = torch.empty_like(q)
    L = torch.empty((B, H), device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream()
    nbytes = 2 * B * Hkv * N * D * 2 + 2 * B * H * D * 2 + B * H * 4
    call = lib.decode if Hkv == H else lib.decode_gqa
    results = {}
    for splits in args.splits:
        for _ in range(max(args.warmup, 3)):
            call(q, K, V, num_splits=splits, O=O, L=L, stream=stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            call(q, K, V, num_splits=splits, O=O, L=L, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        results[splits] = {"ms": ms, "GBps": nbytes / (ms * 1e-3) / 1e9}
    best = max(results, key=lambda s: results[s]["GBps"])
    peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": world * results[best]["GBps"], "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": results[best]["ms"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": ("BASELINE config 4: " if is_config4 else "custom: ") +
                                   (f"split-KV decode B{B} H{H} Nkv{N} D{D}" if Hkv == H else
                                    f"grouped-query split-KV decode B{B} Hq{H} Hkv{Hkv} Nkv{N} D{D}"),
                       "best_num_splits": best},
            "splits": results,
            "roofline": {"bound": "hbm", "achieved": results[best]["GBps"], "peak": peak,
                         "unit": "GB/s", "frac": results[best]["GBps"] / peak,
                         "traffic": traffic_from_profiles("decode") if is_config4 else None},
        }), flush=True)
    return 0


def run_cp(args, lib, dev, world, rank, pk, pk_kind):
    """causal forward over B1 H32 N131072 D128 with ring
    context parallelism across the launched ranks (zigzag shards, NCCL P2P,
    LSE merge)."""
    import torch
    import torch.distributed as dist

    import ring_cp

    B, H, N, D = 1, 32, args.cp_seq, 128
    C = N // (2 * world)
    scale = 1.0 / math.sqrt(D)
    chunks = ring_cp.zigzag_chunks(rank, world)

    def chunk_tensor(kind, c):
        g = torch.Generator(device=dev).manual_seed(41 + 100 * kind + 7919 * c)
        return torch.randn((B, H, C, D), device=dev, generator=g).to(torch.bfloat16)

    q_ab = [chunk_tensor(0, c) for c in chunks]
    k_ab = [chunk_tensor(1, c) for c in chunks]
    v_ab = [chunk_tensor(2, c) for c in chunks]
    do_ab = [chunk_tensor(3, c) for c in chunks] if args.cp_backward else None
    ring = ring_cp.RingAttention(lib)

    def step():
        outs, lses = ring.forward(q_ab, k_ab, v_ab, scale)
        if args.cp_backward:  # the ring backward of the same step
            ring.backward(q_ab, k_ab, v_ab, outs, lses, do_ab, scale)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.index) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = fwd_flops(B, H, N, D, True) * (3.5 if args.cp_backward else 1.0)
    value = flops / (ms * 1e-3) / 1e12
    peak = pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (torch.randn per global chunk)",
            "config": {"workload": f"BASELINE config 5: causal "
                                   f"{'fwd+bwd' if args.cp_backward else 'fwd'} "
                                   f"B{B} H{H} N{N} D{D}, "
                                   f"ring CP over {world} GPU(s), zigzag chunks of {C}",
                       "global_batch": B, "seq_len": N, "parallelism": f"cp{world}"},
            "per_gpu_tflops": value / world,
            "pct_bf16_peak_per_gpu": 100.0 * value / world / peak,
            "clocks": clk.summary(),
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["train", "decode", "cp"], default="train")
    ap.add_argument("--cp-seq", type=int, default=131072)
    ap.add_argument("--cp-backward", action="store_true",
                    help="cp workload: time the ring forward and backward of a training step")
    ap.add_argument("--splits", type=int, nargs="*", default=[0, 1, 2, 4, 8, 16, 32, 64])
    ap.add_argument("--kv-heads", type=int, default=0,
                    help="decode workload: K/V heads (fewer than the 32 query heads: grouped-query)")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
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
