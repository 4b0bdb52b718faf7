"""Split-KV decode, partial forward and log-sum-exp merge on the GPU.

Decode has no reference counterpart; its oracle is the fp64 restatement of
the same formula with one query row, plus a cross-check against the
reference library: the last row of a causal reference forward over
N = kv_len equals decoding that row's query against the whole cache.
"""

import numpy as np
import pytest

import oracle
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu
TOL = 2e-2


def run_decode(lib, q, K, V, dt, scale, splits):
    import torch

    O, L = lib.decode(to_dev(q, dt), to_dev(K, dt), to_dev(V, dt), scale=scale,
                      num_splits=splits)
    torch.cuda.synchronize()
    return host(O), host(L)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("D", [32, 64, 128])
@pytest.mark.parametrize("kv_len,splits", [(1, 0), (7, 1), (300, 3), (1000, 0), (4099, 8),
                                           (5000, 64), (2048, 16)])
def test_decode_vs_f64(lib, cuda, dt, D, kv_len, splits):
    B, H = 2, 3
    q = round_to(oracle.normal((B, H, 1, D), 31 + kv_len), dt)
    K = round_to(oracle.normal((B, H, kv_len, D), 32 + kv_len), dt)
    V = round_to(oracle.normal((B, H, kv_len, D), 33 + kv_len), dt)
    scale = 1.0 / np.sqrt(D)
    O, L = run_decode(lib, q, K, V, dt, scale, splits)
    O64, L64 = oracle.decode_f64(q, K, V, scale)
    assert max_err(O, O64) < TOL
    assert max_err(L, L64) < 1e-3


def test_decode_split_counts_agree(lib, cuda):
    B, H, N, D = 4, 8, 4096, 128
    q = round_to(oracle.normal((B, H, 1, D), 1), "bf16")
    K = round_to(oracle.normal((B, H, N, D), 2), "bf16")
    V = round_to(oracle.normal((B, H, N, D), 3), "bf16")
    base = run_decode(lib, q, K, V, "bf16", 0.088, 1)
    for s in (2, 4, 8, 16, 32, 64):
        O, L = run_decode(lib, q, K, V, "bf16", 0.088, s)
        assert max_err(O, base[0]) < 8e-3
        assert max_err(L, base[1]) < 1e-4


def test_decode_matches_reference_last_row(lib, ref_lib, cuda):
    B, H, N, D = 1, 4, 1024, 128
    Q, K, V = (round_to(oracle.normal((B, H, N, D), s), "bf16") for s in (5, 6, 7))
    scale = 1.0 / np.sqrt(D)
    import torch

    Or, Lr = ref_lib.forward(to_dev(Q, "bf16"), to_dev(K, "bf16"), to_dev(V, "bf16"),
                             causal=True, scale=scale)
    torch.cuda.synchronize()
    O, L = run_decode(lib, Q[:, :, -1:], K, V, "bf16", scale, 0)
    assert max_err(O[:, :, 0], host(Or)[:, :, -1]) < TOL
    assert max_err(L, host(Lr)[:, :, -1]) < 1e-3


def test_config4_decode_sampled(lib, cuda):
    """BASELINE config 4 shape (B64 H32 Nkv16384 D128 bf16); checks sampled units."""
    import torch

    B, H, N, D = 64, 32, 16384, 128
    g = torch.Generator(device="cuda").manual_seed(31)
    q = torch.randn((B, H, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
    O, L = lib.decode(q, K, V, num_splits=0)
    torch.cuda.synchronize()
    for b, h in ((0, 0), (63, 31), (17, 5)):
        sub = [host(x[b:b + 1, h:h + 1]) for x in (q, K, V)]
        O64, L64 = oracle.decode_f64(*sub, 1 / np.sqrt(D))
        assert max_err(host(O[b, h]), O64[0, 0]) < TOL
        assert abs(float(L[b, h]) - L64[0, 0]) < 1e-3
    del K, V


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_partial_forward_with_offsets(lib, cuda, dt):
    import torch

    B, H, Nq, Nk, D = 1, 2, 200, 300, 64
    Q = round_to(oracle.normal((B, H, Nq, D), 1), dt)
    K = round_to(oracle.normal((B, H, Nk, D), 2), dt)
    V = round_to(oracle.normal((B, H, Nk, D), 3), dt)
    for q_off, k_off in [(0, 0), (500, 300), (350, 300), (100, 400), (1000, 0)]:
        O, L = lib.forward_partial(to_dev(Q, dt), to_dev(K, dt), to_dev(V, dt), q_off, k_off,
                                   causal=True, scale=0.125)
        torch.cuda.synchronize()
        O64, L64 = oracle.forward_f64(Q, K, V, 0.125, True, q_off, k_off)
        O, L = host(O), host(L)
        fin = np.isfinite(L64)
        assert np.array_equal(np.isfinite(L), fin)
        assert max_err(O[..., :], O64) < TOL
        assert max_err(L[fin], L64[fin]) < 1e-3


def test_partial_chunks_merge_to_full_forward(lib, cuda):
    """Ring-CP algebra on one GPU: causal attention over N split into 4 chunks
    equals the merge of the per-chunk partials."""
    import torch

    B, H, N, D = 1, 4, 1024, 128
    Q, K, V = (round_to(oracle.normal((B, H, N, D), s), "bf16") for s in (41, 42, 43))
    Qd, Kd, Vd = (to_dev(x, "bf16") for x in (Q, K, V))
    C = N // 4
    O_acc = torch.zeros((B, H, N, D), device="cuda", dtype=torch.float32)
    L_acc = torch.full((B, H, N), float("-inf"), device="cuda", dtype=torch.float32)
    for c in range(4):
        Kc, Vc = Kd[:, :, c * C:(c + 1) * C].contiguous(), Vd[:, :, c * C:(c + 1) * C].contiguous()
        Op, Lp = lib.forward_partial(Qd, Kc, Vc, 0, c * C, causal=True, scale=1 / np.sqrt(D))
        lib.lse_merge(O_acc, L_acc, Op, Lp)
    Ob = torch.empty((B, H, N, D), device="cuda", dtype=torch.bfloat16)
    lib.convert(O_acc, Ob)
    Of, Lf = lib.forward(Qd, Kd, Vd, causal=True, scale=1 / np.sqrt(D))
    torch.cuda.synchronize()
    assert max_err(host(Ob), host(Of)) < 1e-2
    assert max_err(host(L_acc), host(Lf)) < 1e-4
