"""Ring context parallelism on the GPU.

* P ranks emulated in one process on one GPU (no communication: each
  "rank" receives the next owner's K/V payload directly), through the real
  partial-forward / LSE-merge / convert kernels; every rank's output chunks
  must match the single-GPU causal forward over the whole sequence.
* With two or more GPUs: a real two-process ring over NCCL
  (RingAttention, batch_isend_irecv), checked the same way.
"""

import os
import socket

import numpy as np
import pytest

import oracle
import ring_cp
from helpers import host, max_err, round_to, to_dev

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

        ring_cp.run_ring(r, world, C, payload[r], compute_pair, exchange)
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
    emulated on one GPU, equals the single-GPU causal forward."""
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
            pairs = [(qi, ki, chunks[qi] * C, st.k_chunks[ki] * C) for qi, ki in st.pairs]
            for grp in ring_cp.distinct_q_groups(pairs):
                lib.forward_cp_step(Qs, Ks, Vs, O_acc, L_acc, grp, causal=True, scale=scale)
        for qi, c in enumerate(chunks):
            o = torch.empty((B, H, C, D), device="cuda", dtype=torch.bfloat16)
            lib.convert(O_acc[qi], o)
            torch.cuda.synchronize()
            assert max_err(host(o), host(O_full[:, :, c * C:(c + 1) * C])) < 1e-2
            assert max_err(host(L_acc[qi]), host(L_full[:, :, c * C:(c + 1) * C])) < 1e-4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, seed_base, result_dir):
    import torch
    import torch.distributed as dist

    import cuflash_attn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    ok = False
    try:
        lib = cuflash_attn.CuFlashAttn()
        B, H, D, C = 1, 8, 128, 512
        N = 2 * world * C
        g = torch.Generator(device="cuda").manual_seed(seed_base)  # same inputs on every rank
        Q, K, V = (torch.randn((B, H, N, D), device="cuda", generator=g).to(torch.bfloat16)
                   for _ in range(3))
        scale = 1.0 / np.sqrt(D)
        O_full, L_full = lib.forward(Q, K, V, causal=True, scale=scale)
        chunks = ring_cp.zigzag_chunks(rank, world)
        sl = lambda x, c: x[:, :, c * C:(c + 1) * C].contiguous()
        ring = ring_cp.RingAttention(lib)
        outs, lses = ring.forward([sl(Q, c) for c in chunks], [sl(K, c) for c in chunks],
                                  [sl(V, c) for c in chunks], scale)
        torch.cuda.synchronize()
        err_o = max(float((outs[i].float() - sl(O_full, c).float()).abs().max())
                    for i, c in enumerate(chunks))
        err_l = max(float((lses[i] - sl(L_full, c)).abs().max()) for i, c in enumerate(chunks))
        ok = err_o < 1e-2 and err_l < 1e-4
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{err_o} {err_l} {ok}\n")
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_ring_over_nccl_two_gpus(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.start_processes(_nccl_worker, args=(world, _free_port(), 7, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        err_o, err_l, ok = (tmp_path / f"rank{r}.txt").read_text().split()
        assert ok == "True", (r, err_o, err_l)


def test_ring_over_nccl_every_gpu(tmp_path):
    """The same ring over every GPU of the box when it has more than two
    (eight on the BASELINE's CP setting), one rank per GPU."""
    import torch
    import torch.multiprocessing as mp

    world = torch.cuda.device_count()
    if world <= 2:
        pytest.skip("needs more than two GPUs")
    mp.start_processes(_nccl_worker, args=(world, _free_port(), 11, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        err_o, err_l, ok = (tmp_path / f"rank{r}.txt").read_text().split()
        assert ok == "True", (r, err_o, err_l)
