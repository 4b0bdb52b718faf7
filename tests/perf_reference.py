"""Times the reference library (AICL-Lab/cuflash-attn built for sm_100a into
oracle/_ref by `make -C oracle ref`) next to this library on the BASELINE
configs, on the same GPU and inputs, with CUDA events.  Prints one JSON line
per (config, library, pass).  Run on a GPU box:

    python tests/perf_reference.py [--quick]

Not collected by pytest (test infrastructure for the BASELINE.md tables).
"""

import argparse
import json
import math
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "cuflash-attn_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import cuflash_attn  # noqa: E402
import oracle  # noqa: E402

CONFIGS = [
    # name, dtype, B, H, N, D, causal, backward
    ("config1_f32_causal_fwd", torch.float32, 2, 8, 1024, 64, True, False),
    ("f32_causal_fwd_bwd_b2h8n1024d64", torch.float32, 2, 8, 1024, 64, True, True),
    ("f32_fwd_bwd_b4h16n2048d128", torch.float32, 4, 16, 2048, 128, False, True),
    ("config2_f16_fwd_bwd", torch.float16, 4, 16, 2048, 128, False, True),
    ("config3_bf16_causal_fwd_bwd", torch.bfloat16, 8, 32, 4096, 128, True, True),
    ("config5_bf16_causal_fwd_1gpu", torch.bfloat16, 1, 32, 131072, 128, True, False),
]


def timed(fn, iters):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--only", default="", help="substring of the config names to run")
    args = ap.parse_args()
    ours = cuflash_attn.CuFlashAttn()
    ref = cuflash_attn.CuFlashAttn(str(oracle.REF_LIB_PATH), reference_abi_only=True)
    for name, dt, B, H, N, D, causal, bwd in CONFIGS:
        if args.quick and N > 4096:
            continue
        if args.only and args.only not in name:
            continue
        g = torch.Generator(device="cuda").manual_seed(1)
        Q, K, V, dO = (torch.randn((B, H, N, D), device="cuda", generator=g).to(dt)
                       for _ in range(4))
        scale = 1.0 / math.sqrt(D)
        fwd_flop = 4.0 * B * H * N * N * D * (0.5 if causal else 1.0)
        for lname, lib in (("ours", ours), ("reference", ref)):
            O = torch.empty_like(Q)
            L = torch.empty((B, H, N), device="cuda", dtype=torch.float32)
            slow = lname == "reference" and N > 4096
            it = 1 if slow else (2 if lname == "reference" else 20)
            ms = timed(lambda: lib.forward(Q, K, V, causal=causal, scale=scale, O=O, L=L), it)
            print(json.dumps({"config": name, "lib": lname, "pass": "fwd", "ms": ms,
                              "tflops": fwd_flop / ms / 1e9}), flush=True)
            if bwd:
                dQ, dK, dV = (torch.empty_like(Q) for _ in range(3))
                msb = timed(lambda: lib.backward(Q, K, V, O, L, dO, causal=causal, scale=scale,
                                                 dQ=dQ, dK=dK, dV=dV), it)
                print(json.dumps({"config": name, "lib": lname, "pass": "bwd", "ms": msb,
                                  "tflops": 2.5 * fwd_flop / msb / 1e9}), flush=True)
                print(json.dumps({"config": name, "lib": lname, "pass": "fwd+bwd",
                                  "ms": ms + msb,
                                  "tflops": 3.5 * fwd_flop / (ms + msb) / 1e9}), flush=True)


if __name__ == "__main__":
    main()
