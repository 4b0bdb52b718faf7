"""More (batch, head) units than a grid's y dimension holds (65535): the
decode kernels and the fp32 kernels put the units on grid x.  Checked on
sampled units against the fp64 oracle."""

import numpy as np
import pytest

import oracle
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu


def test_decode_more_than_65535_heads(lib, cuda):
    import torch

    B, H, N, D = 2100, 32, 40, 128  # 67200 (b,h) units
    scale = 1.0 / np.sqrt(D)
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
    for splits in (1, 2):
        O, L = lib.decode(q, K, V, scale=scale, num_splits=splits)
        torch.cuda.synchronize()
        assert lib.device_status() == 0
        for b in (0, 1033, B - 1):  # first, middle, last batch entries
            O64, L64 = oracle.decode_f64(host(q[b:b + 1]), host(K[b:b + 1]), host(V[b:b + 1]),
                                         scale)
            assert max_err(host(O[b:b + 1]), O64) < 2e-2
            assert max_err(host(L[b:b + 1]), L64) < 1e-3


def test_grouped_decode_more_than_65535_units(lib, cuda):
    import torch

    B, Hq, Hkv, N, D = 16500, 8, 4, 130, 128  # 66000 (b, K/V head) units
    scale = 1.0 / np.sqrt(D)
    g = torch.Generator(device="cuda").manual_seed(6)
    q = torch.randn((B, Hq, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((B, Hkv, N, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, Hkv, N, D), device="cuda", generator=g).to(torch.bfloat16)
    O, L = lib.decode_gqa(q, K, V, scale=scale)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for b in (0, 8001, B - 1):
        Kr = np.repeat(host(K[b:b + 1]), Hq // Hkv, axis=1)
        Vr = np.repeat(host(V[b:b + 1]), Hq // Hkv, axis=1)
        O64, L64 = oracle.decode_f64(host(q[b:b + 1]), Kr, Vr, scale)
        assert max_err(host(O[b:b + 1]), O64) < 2e-2
        assert max_err(host(L[b:b + 1]), L64) < 1e-3


def test_fp32_forward_backward_more_than_65535_heads(lib, cuda):
    import torch

    B, H, N, D = 66000, 1, 16, 32
    scale = 1.0 / np.sqrt(D)
    g = torch.Generator(device="cuda").manual_seed(7)
    Q, K, V, dO = (torch.randn((B, H, N, D), device="cuda", generator=g) for _ in range(4))
    O, L = lib.forward(Q, K, V, causal=True, scale=scale)
    dQ, dK, dV = lib.backward(Q, K, V, O, L, dO, causal=True, scale=scale)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for b in (0, 40000, B - 1):
        sl = slice(b, b + 1)
        O64, L64 = oracle.forward_f64(host(Q[sl]), host(K[sl]), host(V[sl]), scale, True)
        assert max_err(host(O[sl]), O64) < 1e-4
        gq, gk, gv = oracle.backward_f64(host(Q[sl]), host(K[sl]), host(V[sl]), host(dO[sl]),
                                         scale, True)
        for got, ref in ((dQ, gq), (dK, gk), (dV, gv)):
            assert max_err(host(got[sl]), ref) < 1e-4
