"""Ring context parallelism on the GPU, step by step.

* P ranks emulated in one process on one GPU (no communication: each
  "rank" receives the next owner's K/V payload directly), walking the
  library's ring schedule through the real partial-forward / LSE-merge /
  convert kernels or the one-launch ring-step entry; every rank's output
  chunks must match the single-GPU causal forward over the whole sequence
  and the fp64 oracle on sampled rows.
* The ring entry point itself (cuflash_attention_forward_cp_*, NCCL) is
  tested in test_gpu_ring_cp_nccl.py.
"""

import numpy as np
import pytest

import oracle
import ring_cp
from helpers import host, max_err, round_to, to_dev
from ring_drivers import run_ring

pytestmark = pytest.mark.gpu


def _full_forward(lib, Q, K, V, scale):
    import torch

    O, L = lib.forward(Q, K, V, causal=True, scale=scale)
    torch.cuda.synchronize()
    return O, L


@pytest.mark.parametrize("world", [1, 2, 4, 8])  # 8: the BASELINE CP setting
def test_ring_emulated_on_one_gpu(lib, cuda, world):
    import torch

    B, H, D = 1, 4, 128
    C = 256
    N = 2 * world * C
    Qh, Kh, Vh = (round_to(oracle.normal((B, H, N, D), s), "bf16") for s in (41, 42, 43))
    Q, K, V = (to_dev(x, "bf16") for x in (Qh, Kh, Vh))
    scale = 1.0 / np.sqrt(D)
    O_full, L_full = _full_forward(lib, Q, K, V, scale)
    sl = lambda x, c: x[:, :, c * C:(c + 1) * C].contiguous()
    payload = {}
    for r in range(world):
        ch = ring_cp.zigzag_chunks(r, world)
        payload[r] = torch.stack([torch.stack([sl(K, c) for c in ch]),
                                  torch.stack([sl(V, c) for c in ch])]).contiguous()
    for r in range(world):
        chunks = ring_cp.zigzag_chunks(r, world)
        q_ab = [sl(Q, c) for c in chunks]
        O_acc = [torch.zeros((B, H, C, D), device="cuda") for _ in range(2)]
        L_acc = [torch.full((B, H, C), float("-inf"), device="cuda") for _ in range(2)]
        O_part = torch.empty((B, H, C, D), device="cuda")
        L_part = torch.empty((B, H, C), device="cuda")
        step = {"s": 0}

        def compute_pair(qi, qc, kvbuf, ki, kc):
            lib.forward_partial(q_ab[qi], kvbuf[0, ki], kvbuf[1, ki], qc * C, kc * C,
                                causal=True, scale=scale, O=O_part, L=L_part)
            lib.lse_merge(O_acc[qi], L_acc[qi], O_part, L_part)

        def exchange(cur):
            step["s"] += 1
            owner = ring_cp.kv_owner(r, step["s"], world)
            return lambda: payload[owner]

        run_ring(r, world, payload[r], compute_pair, exchange)
        for qi, c in enumerate(chunks):
            o = torch.empty((B, H, C, D), device="cuda", dtype=torch.bfloat16)
            lib.convert(O_acc[qi], o)
            torch.cuda.synchronize()
            assert max_err(host(o), host(O_full[:, :, c * C:(c + 1) * C])) < 1e-2
            assert max_err(host(L_acc[qi]), host(L_full[:, :, c * C:(c + 1) * C])) < 1e-4


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_cp_step_matches_partial_plus_merge(lib, cuda, D, dt):
    """One multi-pair launch with the in-kernel merge equals separate partial
    forwards folded in with cuflash_lse_merge_f32."""
    import torch

    B, H, C = 1, 4, 320  # C not a multiple of the 256-row q tile
    tdt = torch.bfloat16 if dt == "bf16" else torch.float16
    g = torch.Generator(device="cuda").manual_seed(5)
    Q = torch.randn((2, B, H, C, D), device="cuda", generator=g).to(tdt)
    K = torch.randn((3, B, H, C, D), device="cuda", generator=g).to(tdt)
    V = torch.randn((3, B, H, C, D), device="cuda", generator=g).to(tdt)
    scale = 1.0 / np.sqrt(D)
    # running state from an earlier step: slot 0 holds a merged result, slot 1 is empty
    O0 = torch.randn((2, B, H, C, D), device="cuda", generator=g) * 0.1
    L0 = torch.randn((2, B, H, C), device="cuda", generator=g)
    O0[1].zero_()
    L0[1].fill_(float("-inf"))
    steps = [
        [(0, 2, 5 * C, 1 * C), (1, 0, 2 * C, 2 * C)],  # fully visible; diagonal
        [(1, 1, 2 * C, 3 * C)],                         # fully masked (keys after queries)
        [(0, 1, 5 * C, 5 * C), (1, 2, 2 * C, 0)],        # diagonal; fully visible
    ]
    Oa, La = O0.clone(), L0.clone()
    Ob, Lb = O0.clone(), L0.clone()
    for pairs in steps:
        lib.forward_cp_step(Q, K, V, Oa, La, pairs, causal=True, scale=scale)
        for qs, ks, qo, ko in pairs:
            Op, Lp = lib.forward_partial(Q[qs], K[ks], V[ks], qo, ko, causal=True, scale=scale)
            lib.lse_merge(Ob[qs], Lb[qs], Op, Lp)
    torch.cuda.synchronize()
    assert torch.allclose(Oa, Ob, rtol=1e-5, atol=1e-6), float((Oa - Ob).abs().max())
    fin = torch.isfinite(Lb)
    assert torch.equal(fin, torch.isfinite(La))
    assert torch.allclose(La[fin], Lb[fin], rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("world", [1, 2, 4, 8])  # 8: the BASELINE CP setting
def test_ring_cp_step_emulated_on_one_gpu(lib, cuda, world):
    """The ring schedule through the single-launch step entry, P ranks
    emulated on one GPU, equals the single-GPU causal forward and, on every
    7th query row, the fp64 oracle."""
    import torch

    B, H, D = 1, 4, 128
    C = 256
    N = 2 * world * C
    Qh, Kh, Vh = (round_to(oracle.normal((B, H, N, D), s), "bf16") for s in (41, 42, 43))
    Q, K, V = (to_dev(x, "bf16") for x in (Qh, Kh, Vh))
    scale = 1.0 / np.sqrt(D)
    O_full, L_full = _full_forward(lib, Q, K, V, scale)
    sl = lambda x, c: x[:, :, c * C:(c + 1) * C].contiguous()
    stack = lambda x, cs: torch.stack([sl(x, c) for c in cs]).contiguous()
    for r in range(world):
        chunks = ring_cp.zigzag_chunks(r, world)
        Qs = stack(Q, chunks)
        O_acc = torch.zeros((2, B, H, C, D), device="cuda")
        L_acc = torch.full((2, B, H, C), float("-inf"), device="cuda")
        for st in ring_cp.ring_steps(r, world):
            Ks, Vs = stack(K, st.k_chunks), stack(V, st.k_chunks)
            for launch in st.launches:
                grp = [(qi, ki, chunks[qi] * C, st.k_chunks[ki] * C) for qi, ki in launch]
                lib.forward_cp_step(Qs, Ks, Vs, O_acc, L_acc, grp, causal=True, scale=scale)
        for qi, c in enumerate(chunks):
            o = torch.empty((B, H, C, D), device="cuda", dtype=torch.bfloat16)
            lib.convert(O_acc[qi], o)
            torch.cuda.synchronize()
            assert max_err(host(o), host(O_full[:, :, c * C:(c + 1) * C])) < 1e-2
            assert max_err(host(L_acc[qi]), host(L_full[:, :, c * C:(c + 1) * C])) < 1e-4
            rows = np.arange(c * C, (c + 1) * C, 7)
            O64, L64 = oracle.forward_rows_f64(Qh, Kh, Vh, scale, True, rows)
            assert max_err(host(o)[:, :, rows - c * C], O64) < 2e-2
            assert max_err(host(L_acc[qi])[:, :, rows - c * C], L64) < 1e-3
