"""The allocation-free split-KV decode entry point
(cuflash_attention_decode_bf16_noalloc), called through the C ABI and
checked against the regular decode entry point.

Who needs it: callers that must not have device memory allocated on their
behalf, such as a serving engine that has already claimed nearly all of HBM
for its KV-cache pages (a library allocation would fail or fragment that
reservation) or a per-token decode loop that keeps allocation calls, with
their unpredictable cost, out of its hot path.  The entry point keeps its
split partials in a fixed device buffer instead.

This file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest

import cuflash_attn as cf
import oracle

pytestmark = pytest.mark.gpu

TOL_O = 2e-2  # the decode tests' tolerance on O
TOL_L = 1e-3  # ... and on the log-sum-exp


def _noalloc(lib, q, K, V, O, L, splits):
    import torch

    B, H, N, D = K.shape
    fn = lib.lib.cuflash_attention_decode_bf16_noalloc
    return fn(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(K.data_ptr()),
              ctypes.c_void_p(V.data_ptr()), ctypes.c_void_p(O.data_ptr()),
              ctypes.c_void_p(L.data_ptr()), B, H, N, D, ctypes.c_float(D ** -0.5), splits,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _inputs(B, H, N, D, seed):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
    return q, K, V


def test_noalloc_decode_matches_regular_decode_on_consecutive_calls(lib, cuda):
    import torch

    # two calls in a row, different shapes and split counts: the second call
    # runs on whatever the first left in the shared buffer
    for B, H, N, D, splits, seed in [(4, 8, 4096, 128, 8, 1), (2, 16, 3000, 64, 16, 2),
                                     (4, 8, 4096, 128, 0, 3)]:
        q, K, V = _inputs(B, H, N, D, seed)
        O_ref, L_ref = lib.decode(q, K, V, scale=D ** -0.5, num_splits=splits)
        O = torch.full_like(O_ref, float("nan"))
        L = torch.full_like(L_ref, float("nan"))
        assert _noalloc(lib, q, K, V, O, L, splits) == cf.SUCCESS
        torch.cuda.synchronize()
        assert torch.isfinite(O.float()).all() and torch.isfinite(L).all()
        assert (O.float() - O_ref.float()).abs().max().item() < TOL_O
        assert (L - L_ref).abs().max().item() < TOL_L


def test_noalloc_decode_rejects_splits_beyond_its_buffer(lib, cuda):
    import torch

    # 8*32 heads * 64 splits * (128 + 1) fp32 values exceed the 8 MiB buffer
    q, K, V = _inputs(8, 32, 2048, 128, 4)
    O = torch.empty_like(q)
    L = torch.empty((8, 32), device="cuda", dtype=torch.float32)
    assert _noalloc(lib, q, K, V, O, L, 64) == cf.OUT_OF_MEMORY
    # the same problem with a split count that fits still works
    assert _noalloc(lib, q, K, V, O, L, 4) == cf.SUCCESS
    torch.cuda.synchronize()
    O_ref, L_ref = lib.decode(q, K, V, scale=128 ** -0.5, num_splits=4)
    torch.cuda.synchronize()
    assert (O.float() - O_ref.float()).abs().max().item() < TOL_O


def test_noalloc_decode_against_fp64(lib, cuda):
    """Directly against the fp64 oracle (not only through the regular decode),
    twice in a row, with an explicit split count and with the automatic one at
    a large batch (B64 H32: 2048 heads share the buffer; with 148 SMs the
    automatic split count, about 4 CTAs per SM, stays far below the 8 MiB
    limit, so the cap on it never binds)."""
    import torch

    for B, H, N, D, splits, seed in [(2, 4, 2500, 128, 8, 11), (64, 32, 1024, 128, 0, 12)]:
        q, K, V = _inputs(B, H, N, D, seed)
        O = torch.full_like(q, float("nan"))
        L = torch.full((B, H), float("nan"), device="cuda", dtype=torch.float32)
        for _ in range(2):
            assert _noalloc(lib, q, K, V, O, L, splits) == cf.SUCCESS
            torch.cuda.synchronize()
            heads = [(0, 0), (B - 1, H - 1), (B // 2, H // 3)]
            for b, h in heads:
                qh = q[b:b + 1, h:h + 1].float().cpu().numpy()
                Kh = K[b:b + 1, h:h + 1].float().cpu().numpy()
                Vh = V[b:b + 1, h:h + 1].float().cpu().numpy()
                O64, L64 = oracle.decode_f64(qh, Kh, Vh, D ** -0.5)
                got_o = O[b, h].float().cpu().numpy().reshape(O64.shape)
                got_l = L[b, h].cpu().numpy().reshape(L64.shape)
                assert np.max(np.abs(got_o - O64)) < TOL_O
                assert np.max(np.abs(got_l - L64)) < TOL_L
