"""Grouped-query attention with separate query / key lengths on the GPU
(cuflash_attention_{forward,backward}_gqa_*), against the fp64 oracle with
K/V heads repeated per group and the bottom-right causal alignment
(query i sees key j iff j <= i + Nk - Nq).

Bars: fp16/bf16 within 2e-2 of fp64 (the reference tests' low-precision
tolerance); with one query head per K/V head and equal lengths the forward
equals the reference-ABI forward bit for bit and the backward stays within
one output ulp of it.
"""

import numpy as np
import pytest

import oracle
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu

TOL = 2e-2

SHAPES = [
    # B, Hq, Hkv, Nq, Nk, D, causal
    (2, 8, 2, 128, 384, 128, True),     # group 4, fewer queries than keys
    (1, 6, 1, 300, 140, 64, True),      # MQA, more queries than keys (first rows see nothing)
    (1, 4, 2, 257, 513, 128, False),    # ragged lengths, non-causal
    (1, 8, 8, 1, 1000, 128, True),      # one query row against a 1000-key cache
    (2, 4, 4, 200, 200, 32, True),      # equal lengths, MHA
    (1, 4, 2, 200, 456, 64, True),      # offset not a multiple of 128
]


def _inputs(shape, dt, seed):
    B, Hq, Hkv, Nq, Nk, D, _ = shape
    Q = round_to(oracle.normal((B, Hq, Nq, D), seed), dt)
    K = round_to(oracle.normal((B, Hkv, Nk, D), seed + 1), dt)
    V = round_to(oracle.normal((B, Hkv, Nk, D), seed + 2), dt)
    dO = round_to(oracle.normal((B, Hq, Nq, D), seed + 3), dt)
    return Q, K, V, dO


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:6])) + ("c" if s[6] else "n"))
def test_gqa_forward_backward_vs_fp64(lib, cuda, shape, dt):
    import torch

    B, Hq, Hkv, Nq, Nk, D, causal = shape
    scale = 1.0 / np.sqrt(D)
    Qh, Kh, Vh, dOh = _inputs(shape, dt, 100 + Nq)
    Q, K, V, dO = (to_dev(x, dt) for x in (Qh, Kh, Vh, dOh))
    O, L = lib.forward_gqa(Q, K, V, causal=causal, scale=scale)
    dQ, dK, dV = lib.backward_gqa(Q, K, V, O, L, dO, causal=causal, scale=scale)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    O64, L64 = oracle.gqa_forward_f64(Qh, Kh, Vh, scale, causal)
    assert max_err(host(O), O64) < TOL
    Lg = host(L)
    fin = np.isfinite(L64)
    assert np.array_equal(np.isfinite(Lg), fin)          # rows without keys: L = -inf
    assert max_err(Lg[fin], L64[fin]) < 1e-3
    if not fin.all():
        assert np.all(host(O)[~fin] == 0.0)
    dQ64, dK64, dV64 = oracle.gqa_backward_f64(Qh, Kh, Vh, dOh, scale, causal)
    for got, ref in ((dQ, dQ64), (dK, dK64), (dV, dV64)):
        g = host(got)
        assert np.all(np.isfinite(g))
        assert max_err(g, ref) < TOL * max(1.0, float(np.abs(ref).max()))


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_gqa_with_one_group_matches_reference_abi(lib, cuda, dt):
    import torch

    B, H, N, D = 2, 4, 333, 128
    scale = 1.0 / np.sqrt(D)
    Qh, Kh, Vh, dOh = _inputs((B, H, H, N, N, D, True), dt, 7)
    Q, K, V, dO = (to_dev(x, dt) for x in (Qh, Kh, Vh, dOh))
    O1, L1 = lib.forward(Q, K, V, causal=True, scale=scale)
    O2, L2 = lib.forward_gqa(Q, K, V, causal=True, scale=scale)
    torch.cuda.synchronize()
    assert torch.equal(O1, O2) and torch.equal(L1, L2)
    g1 = lib.backward(Q, K, V, O1, L1, dO, causal=True, scale=scale)
    g2 = lib.backward_gqa(Q, K, V, O1, L1, dO, causal=True, scale=scale)
    torch.cuda.synchronize()
    for a, b in zip(g1, g2):
        # dQ sums per-block contributions with atomics: order may differ
        assert max_err(host(a), host(b)) <= 2.0 ** (np.floor(np.log2(float(a.float().abs().max()))) - 7)


@pytest.mark.parametrize("dt", ["bf16"])
def test_gqa_forward_equals_repeated_heads(lib, cuda, dt):
    """Group 4: the same result as the reference-ABI forward on K/V heads
    repeated per group (the kernels read the same values)."""
    import torch

    B, Hq, Hkv, N, D = 1, 8, 2, 512, 128
    Qh, Kh, Vh, _ = _inputs((B, Hq, Hkv, N, N, D, True), dt, 11)
    Q, K, V = (to_dev(x, dt) for x in (Qh, Kh, Vh))
    O1, L1 = lib.forward_gqa(Q, K, V, causal=True)
    Kr = K.repeat_interleave(Hq // Hkv, dim=1).contiguous()
    Vr = V.repeat_interleave(Hq // Hkv, dim=1).contiguous()
    O2, L2 = lib.forward(Q, Kr, Vr, causal=True)
    torch.cuda.synchronize()
    assert torch.equal(O1, O2) and torch.equal(L1, L2)
