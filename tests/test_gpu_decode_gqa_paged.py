"""Grouped-query and paged-KV split-KV decode on the GPU
(cuflash_attention_decode_{gqa,paged}_*), against the fp64 oracle on the
same inputs (K/V heads repeated per group; pages gathered into a contiguous
cache per sequence).

Bars: fp16/bf16 O within 2e-2 of fp64 and L within 1e-3 (the decode tests'
bars); the grouped kernel with one head per group agrees with the MHA decode
entry point to rounding.
"""

import numpy as np
import pytest

import oracle
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu

TOL_O = 2e-2
TOL_L = 1e-3


def _ref_decode(q, K, V, scale):
    """q [B,Hq,1,D], K/V [B,Hkv,N,D] -> fp64 O [B,Hq,1,D], L [B,Hq]."""
    g = q.shape[1] // K.shape[1]
    return oracle.decode_f64(q, np.repeat(K, g, axis=1), np.repeat(V, g, axis=1), scale)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (8, 4), (16, 4), (32, 4), (12, 2), (14, 2), (7, 1)])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_decode_gqa_vs_fp64(lib, cuda, dt, Hq, Hkv, splits, D):
    """Head_dim 64 and 128 take the tensor-core kernel from two heads per
    K/V head up, the SIMT kernel for one."""
    import torch

    B, N = 2, 777
    scale = 1.0 / np.sqrt(D)
    q = round_to(oracle.normal((B, Hq, 1, D), 1), dt)
    K = round_to(oracle.normal((B, Hkv, N, D), 2), dt)
    V = round_to(oracle.normal((B, Hkv, N, D), 3), dt)
    O, L = lib.decode_gqa(to_dev(q, dt), to_dev(K, dt), to_dev(V, dt), scale=scale,
                          num_splits=splits)
    torch.cuda.synchronize()
    O64, L64 = _ref_decode(q, K, V, scale)
    assert max_err(host(O), O64) < TOL_O
    assert max_err(host(L), L64) < TOL_L


@pytest.mark.parametrize("D", [32, 64])
def test_decode_gqa_head_dims(lib, cuda, D):
    import torch

    B, Hq, Hkv, N = 3, 8, 2, 300
    scale = 1.0 / np.sqrt(D)
    q = round_to(oracle.normal((B, Hq, 1, D), 4), "bf16")
    K = round_to(oracle.normal((B, Hkv, N, D), 5), "bf16")
    V = round_to(oracle.normal((B, Hkv, N, D), 6), "bf16")
    O, L = lib.decode_gqa(to_dev(q, "bf16"), to_dev(K, "bf16"), to_dev(V, "bf16"), scale=scale)
    torch.cuda.synchronize()
    O64, L64 = _ref_decode(q, K, V, scale)
    assert max_err(host(O), O64) < TOL_O and max_err(host(L), L64) < TOL_L


def test_decode_gqa_group_one_matches_mha_decode(lib, cuda):
    import torch

    B, H, N, D = 4, 8, 1000, 128
    q, K, V = (to_dev(round_to(oracle.normal(s, seed), "bf16"), "bf16")
               for s, seed in (((B, H, 1, D), 7), ((B, H, N, D), 8), ((B, H, N, D), 9)))
    O1, L1 = lib.decode(q, K, V)
    O2, L2 = lib.decode_gqa(q, K, V)
    torch.cuda.synchronize()
    assert max_err(host(O1), host(O2)) <= 2.0 ** -8
    assert max_err(host(L1), host(L2)) < 1e-5


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("page_size,Hq,Hkv", [(16, 8, 2), (64, 4, 4), (128, 32, 8), (1, 4, 1)])
@pytest.mark.parametrize("splits", [0, 2])
def test_decode_paged_vs_fp64(lib, cuda, dt, page_size, Hq, Hkv, splits, D):
    import torch

    B = 5
    max_pages = max(1, 700 // page_size + 2)
    num_pages = B * max_pages + 3
    rng = np.random.default_rng(page_size + Hq)
    seq_lens = np.array([0, 1, page_size * 3 + 5, 650, max_pages * page_size], np.int32)[:B]
    seq_lens = np.minimum(seq_lens, max_pages * page_size).astype(np.int32)
    table = rng.permutation(num_pages)[:B * max_pages].reshape(B, max_pages).astype(np.int32)
    q = round_to(oracle.normal((B, Hq, 1, D), 11), dt)
    Kc = round_to(oracle.normal((num_pages, page_size, Hkv, D), 12), dt)
    Vc = round_to(oracle.normal((num_pages, page_size, Hkv, D), 13), dt)
    scale = 1.0 / np.sqrt(D)
    O, L = lib.decode_paged(to_dev(q, dt), to_dev(Kc, dt), to_dev(Vc, dt),
                            torch.from_numpy(table).cuda(), torch.from_numpy(seq_lens).cuda(),
                            scale=scale, num_splits=splits)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    Og, Lg = host(O), host(L)
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            assert np.all(Og[b] == 0.0) and np.all(np.isneginf(Lg[b]))
            continue
        t = np.arange(n)
        rows = table[b, t // page_size] * page_size + t % page_size
        Kb = Kc.reshape(-1, Hkv, D)[rows].transpose(1, 0, 2)[None]  # [1, Hkv, n, D]
        Vb = Vc.reshape(-1, Hkv, D)[rows].transpose(1, 0, 2)[None]
        O64, L64 = _ref_decode(q[b:b + 1], Kb, Vb, scale)
        assert max_err(Og[b:b + 1], O64) < TOL_O, b
        assert max_err(Lg[b:b + 1], L64) < TOL_L, b


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("tc", ["1", "0"])
@pytest.mark.parametrize("Hq,Hkv", [(48, 2), (64, 2), (4, 2)])
def test_decode_gqa_large_groups_and_rescale(lib, cuda, tc, Hq, Hkv, D):
    """Groups above 16 heads (several head tiles per K/V head on the tensor-
    core path) and scores that grow along the cache (later rows dominate,
    so running maxima rise across blocks and O is rescaled), on both the
    tensor-core kernel (CUFLASH_DECODE_GQA_TC=1, head_dim 64 and 128) and the
    SIMT kernel (=0)."""
    lib.set_option("CUFLASH_DECODE_GQA_TC", int(tc))
    try:
        _check_large_groups(lib, Hq, Hkv, D)
    finally:
        lib.set_option("CUFLASH_DECODE_GQA_TC", -1)


def _check_large_groups(lib, Hq, Hkv, D):
    import torch

    B, N, dt = 2, 1500, "bf16"
    scale = 1.0 / np.sqrt(D)
    q = round_to(oracle.normal((B, Hq, 1, D), 21), dt)
    ramp = (1.0 + 4.0 * np.arange(N, dtype=np.float32) / N)[None, None, :, None]
    K = round_to(oracle.normal((B, Hkv, N, D), 22) * ramp, dt)
    V = round_to(oracle.normal((B, Hkv, N, D), 23), dt)
    for splits in (0, 1):
        O, L = lib.decode_gqa(to_dev(q, dt), to_dev(K, dt), to_dev(V, dt), scale=scale,
                              num_splits=splits)
        torch.cuda.synchronize()
        assert lib.device_status() == 0
        O64, L64 = _ref_decode(q, K, V, scale)
        assert max_err(host(O), O64) < TOL_O
        assert max_err(host(L), L64) < TOL_L
