"""Ring context parallelism on CPU: the library's ring schedule
(cuflash_cp_ring_schedule, the host function libcuflash_attn_cp.so's NCCL
ring follows) and the multi-process ring (world_size 2 to 4, gloo) walking
that schedule with the fp64 oracle standing in for the GPU kernels, forward
and backward.  The assembled result must equal full attention (and its
gradients) over the whole sequence."""

import ctypes


import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cuflash_attn as cf
import oracle
import ring_cp
from ring_drivers import run_ring, run_ring_backward


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_schedule_covers_every_visible_pair_once(world):
    seen = {}
    for r in range(world):
        q_chunks = ring_cp.zigzag_chunks(r, world)
        for st in ring_cp.ring_steps(r, world):
            for qi, ki in st.pairs:
                key = (q_chunks[qi], st.k_chunks[ki])
                seen[key] = seen.get(key, 0) + 1
    expected = {(q, k) for q in range(2 * world) for k in range(q + 1)}
    assert set(seen) == expected
    assert all(v == 1 for v in seen.values())
    # zigzag balances the causal work: every rank sees the same number of
    # (query chunk, key chunk) pairs, counting diagonal ones as half
    work = []
    for r in range(world):
        qc = ring_cp.zigzag_chunks(r, world)
        work.append(sum((0.5 if k == q else 1.0) for q in qc for k in range(q + 1)))
    assert max(work) == min(work)


@pytest.mark.parametrize("causal", [True, False])
def test_forward_launch_groups(causal):
    """A forward launch merges every query slot at most once; every step
    needs at most two launches and covers each of its pairs once."""
    for world in (1, 2, 3, 8):
        for r in range(world):
            for st in ring_cp.ring_steps(r, world, causal):
                for g in st.launches:
                    assert len({qi for qi, _ in g}) == len(g)
                assert sorted(p for g in st.launches for p in g) == sorted(st.pairs)
                assert len(st.launches) <= 2
                if not causal:
                    assert len(st.pairs) == 4


def test_non_causal_schedule_covers_every_pair():
    world = 3
    seen = set()
    for r in range(world):
        qc = ring_cp.zigzag_chunks(r, world)
        for st in ring_cp.ring_steps(r, world, causal=False):
            seen |= {(qc[qi], st.k_chunks[ki]) for qi, ki in st.pairs}
    assert seen == {(q, k) for q in range(2 * world) for k in range(2 * world)}


def test_schedule_validation():
    lib = ring_cp.load_cp_library()
    out = [ctypes.c_int() for _ in range(2)]
    arrs = [(ctypes.c_int * 4)() for _ in range(5)]
    call = lambda r, w, s, nul=False: lib.cuflash_cp_ring_schedule(
        r, w, s, True, None if nul else ctypes.byref(out[0]), ctypes.byref(out[1]),
        *[ctypes.cast(a, ctypes.c_void_p) for a in arrs])
    assert call(0, 2, 0) == cf.SUCCESS
    assert call(0, 2, 0, nul=True) == cf.NULL_POINTER
    assert call(2, 2, 0) == cf.INVALID_DIMENSION      # rank outside [0, world)
    assert call(0, 2, 2) == cf.INVALID_DIMENSION      # step outside [0, world)
    assert call(0, 0, 0) == cf.INVALID_DIMENSION


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, Q, K, V, scale, out_path, causal=True):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, N, D = Q.shape
        C = N // (2 * world)
        chunks = ring_cp.zigzag_chunks(rank, world)
        sl = lambda x, c: np.ascontiguousarray(x[:, :, c * C:(c + 1) * C])
        q_local = [sl(Q, c) for c in chunks]
        kv = torch.from_numpy(np.stack([np.stack([sl(K, c) for c in chunks]),
                                        np.stack([sl(V, c) for c in chunks])]))
        O_acc = [np.zeros((B, H, C, D)) for _ in range(2)]
        L_acc = [np.full((B, H, C), -np.inf) for _ in range(2)]

        def compute_pair(qi, qc, kvbuf, ki, kc):
            kb = kvbuf.numpy()
            Op, Lp = oracle.forward_f64(q_local[qi], kb[0, ki], kb[1, ki], scale, causal,
                                        q_offset=qc * C, k_offset=kc * C)
            M = np.maximum(L_acc[qi], Lp)
            fin = np.isfinite(M)
            wa = np.where(fin, np.exp(np.where(fin, L_acc[qi] - M, 0)), 0.0)
            wb = np.where(fin, np.exp(np.where(fin, Lp - M, 0)), 0.0)
            tot = wa + wb
            safe = np.where(tot > 0, tot, 1.0)
            O_acc[qi] = (wa[..., None] * O_acc[qi] + wb[..., None] * Op) / safe[..., None]
            L_acc[qi] = np.where(tot > 0, M + np.log(safe), -np.inf)

        def exchange(cur):
            nxt = torch.empty_like(cur)
            reqs = [dist.isend(cur, (rank + 1) % world), dist.irecv(nxt, (rank - 1) % world)]

            def wait():
                for r in reqs:
                    r.wait()
                return nxt

            return wait

        run_ring(rank, world, kv, compute_pair, exchange, causal)
        np.savez(out_path + f".{rank}.npz", O0=O_acc[0], O1=O_acc[1], L0=L_acc[0], L1=L_acc[1])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,causal", [(2, True), (3, True), (4, True), (2, False)])
def test_ring_over_gloo_equals_full_attention(world, causal, tmp_path):
    B, H, D = 1, 2, 32
    N = 2 * world * 12
    Q, K, V = (oracle.uniform((B, H, N, D), s) for s in (5, 6, 7))
    scale = 1.0 / np.sqrt(D)
    out = str(tmp_path / "ring")
    mp.start_processes(_worker, args=(world, _free_port(), Q, K, V, scale, out, causal),
                       nprocs=world, join=True, start_method="spawn")
    O_full, L_full = oracle.forward_f64(Q, K, V, scale, causal)
    C = N // (2 * world)
    for r in range(world):
        res = np.load(out + f".{r}.npz")
        for slot, c in enumerate(ring_cp.zigzag_chunks(r, world)):
            np.testing.assert_allclose(res[f"O{slot}"], O_full[:, :, c * C:(c + 1) * C],
                                       atol=1e-10)
            np.testing.assert_allclose(res[f"L{slot}"], L_full[:, :, c * C:(c + 1) * C],
                                       atol=1e-10)


def test_backward_pairs_sum_to_full_backward():
    """The per-pair backward with the full-row statistics, summed over the
    zigzag ring's pairs, is the full causal backward."""
    B, H, D, world = 1, 2, 16, 3
    C = 10
    N = 2 * world * C
    Q, K, V, dO = (oracle.uniform((B, H, N, D), s) for s in (11, 12, 13, 14))
    scale = 1.0 / np.sqrt(D)
    O, L = oracle.forward_f64(Q, K, V, scale, True)
    Dv = (dO.astype(np.float64) * O).sum(-1)
    dQ = np.zeros((B, H, N, D))
    dK = np.zeros((B, H, N, D))
    dV = np.zeros((B, H, N, D))
    sl = lambda c: slice(c * C, (c + 1) * C)
    for r in range(world):
        qc = ring_cp.zigzag_chunks(r, world)
        for st in ring_cp.ring_steps(r, world):
            for qi, ki in st.pairs:
                a, b = qc[qi], st.k_chunks[ki]
                gq, gk, gv = oracle.backward_pair_f64(
                    Q[:, :, sl(a)], K[:, :, sl(b)], V[:, :, sl(b)], dO[:, :, sl(a)],
                    L[:, :, sl(a)], Dv[:, :, sl(a)], scale, True, a * C, b * C)
                dQ[:, :, sl(a)] += gq
                dK[:, :, sl(b)] += gk
                dV[:, :, sl(b)] += gv
    rQ, rK, rV = oracle.backward_f64(Q, K, V, dO, scale, True)
    for got, ref in ((dQ, rQ), (dK, rK), (dV, rV)):
        np.testing.assert_allclose(got, ref, atol=1e-10)


@pytest.mark.parametrize("world", [1, 2, 5])
def test_dkv_hops_return_home(world):
    for r in range(world):
        hops = ring_cp.dkv_hops(r, world)
        assert hops[0] == r                           # step 0: own K/V
        assert (r + 1) % world == hops[-1]            # the last send reaches its owner
    # every owner's accumulator visits every rank exactly once
    for o in range(world):
        visits = [r for r in range(world) for s, h in enumerate(ring_cp.dkv_hops(r, world))
                  if h == o]
        assert sorted(visits) == list(range(world))


def _bwd_worker(rank, world, port, Q, K, V, dO, scale, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, N, D = Q.shape
        C = N // (2 * world)
        chunks = ring_cp.zigzag_chunks(rank, world)
        sl = lambda x, c: np.ascontiguousarray(x[:, :, c * C:(c + 1) * C])
        # the forward's statistics of this rank's rows (the ring forward's output)
        O, L = oracle.forward_f64(Q, K, V, scale, True)
        Dv = (dO.astype(np.float64) * O).sum(-1)
        kv = torch.from_numpy(np.stack([np.stack([sl(K, c) for c in chunks]),
                                        np.stack([sl(V, c) for c in chunks])]))
        dq = [np.zeros((B, H, C, D)) for _ in range(2)]

        def compute_step(st, kvbuf, acc):
            kb = kvbuf.numpy()
            for qi, ki in st.pairs:
                qc, kc = chunks[qi], st.k_chunks[ki]
                gq, gk, gv = oracle.backward_pair_f64(sl(Q, qc), kb[0, ki], kb[1, ki],
                                                      sl(dO, qc), sl(L, qc), sl(Dv, qc), scale,
                                                      True, qc * C, kc * C)
                dq[qi] += gq
                acc[0, ki] += torch.from_numpy(gk)
                acc[1, ki] += torch.from_numpy(gv)

        def exchange(cur):
            nxt = torch.empty_like(cur)
            reqs = [dist.isend(cur, (rank + 1) % world), dist.irecv(nxt, (rank - 1) % world)]

            def wait():
                for r in reqs:
                    r.wait()
                return nxt

            return wait

        acc = run_ring_backward(
            rank, world, kv, compute_step, exchange,
            lambda: torch.zeros((2, 2, B, H, C, D), dtype=torch.float64),
            lambda a, b: a + b)
        a = acc.numpy()
        np.savez(out_path + f".{rank}.npz", dQ0=dq[0], dQ1=dq[1], dK0=a[0, 0], dK1=a[0, 1],
                 dV0=a[1, 0], dV1=a[1, 1])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_ring_backward_over_gloo_equals_full_backward(world, tmp_path):
    B, H, D = 1, 2, 16
    N = 2 * world * 8
    Q, K, V, dO = (oracle.uniform((B, H, N, D), s) for s in (21, 22, 23, 24))
    scale = 1.0 / np.sqrt(D)
    out = str(tmp_path / "ringb")
    mp.start_processes(_bwd_worker, args=(world, _free_port(), Q, K, V, dO, scale, out),
                       nprocs=world, join=True, start_method="spawn")
    rQ, rK, rV = oracle.backward_f64(Q, K, V, dO, scale, True)
    C = N // (2 * world)
    for r in range(world):
        res = np.load(out + f".{r}.npz")
        for slot, c in enumerate(ring_cp.zigzag_chunks(r, world)):
            sl = slice(c * C, (c + 1) * C)
            np.testing.assert_allclose(res[f"dQ{slot}"], rQ[:, :, sl], atol=1e-10)
            np.testing.assert_allclose(res[f"dK{slot}"], rK[:, :, sl], atol=1e-10)
            np.testing.assert_allclose(res[f"dV{slot}"], rV[:, :, sl], atol=1e-10)


@pytest.mark.parametrize("sfx", ["bf16", "f16"])
def test_ring_entry_validation(sfx):
    """cuflash_attention_{forward,backward}_cp_*: argument checks happen
    before any CUDA or NCCL call, in the reference's order (null pointers,
    sizes, head_dim, scale), so they run on a machine without a GPU."""
    lib = ring_cp.load_cp_library()
    fake, nul = ctypes.c_void_p(0x10000), ctypes.c_void_p(0)
    comm = ctypes.c_void_p(0x20000)  # never dereferenced: every call below fails validation
    fwd = getattr(lib, f"cuflash_attention_forward_cp_{sfx}")
    bwd = getattr(lib, f"cuflash_attention_backward_cp_{sfx}")

    def f(nul_at=None, B=1, H=2, N=512, D=64, scale=0.1, comm_=comm, rank=0, world=2,
          reserve=-1):
        a = [fake] * 5 + [B, H, N, D, scale, True, comm_, rank, world, reserve, nul]
        if nul_at is not None:
            a[nul_at] = nul
        return fwd(*a)

    def b(nul_at=None, **kw):
        a = [fake] * 9 + [1, 2, 512, kw.get("D", 64), 0.1, True, comm, 0, kw.get("world", 2),
                          -1, nul]
        if nul_at is not None:
            a[nul_at] = nul
        return bwd(*a)

    assert f(nul_at=0) == cf.NULL_POINTER and f(nul_at=4) == cf.NULL_POINTER
    assert f(B=0) == cf.INVALID_DIMENSION and f(N=-4) == cf.INVALID_DIMENSION
    assert f(N=510) == cf.INVALID_DIMENSION           # not a multiple of 2 * world
    assert f(world=0) == cf.INVALID_DIMENSION and f(rank=2) == cf.INVALID_DIMENSION
    assert f(world=257, N=257 * 2 * 4) == cf.INVALID_DIMENSION
    assert f(reserve=-2) == cf.INVALID_DIMENSION
    assert f(D=80) == cf.UNSUPPORTED_HEAD_DIM
    assert f(scale=-1.0) == cf.INVALID_DIMENSION and f(scale=float("inf")) == cf.INVALID_DIMENSION
    assert f(comm_=nul) == cf.NULL_POINTER             # several ranks need a communicator
    # the reference's backward order: gradient pointers first
    assert b(nul_at=5) == cf.NULL_POINTER and b(nul_at=8) == cf.NULL_POINTER
    assert b(nul_at=0) == cf.NULL_POINTER
    assert b(D=48) == cf.UNSUPPORTED_HEAD_DIM
    assert b(world=0) == cf.INVALID_DIMENSION


def _leaving_worker(rank, world, port, out_path, leave_rank, leave_after):
    """One ring rank over gloo with a short timeout; rank `leave_rank` leaves
    (exits without tearing anything down) between ring steps, after
    `leave_after` steps.  The others record how their next exchange ended."""
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    B, H, C, D = 1, 1, 8, 16
    kv = torch.zeros((2, 2, B, H, C, D), dtype=torch.float64)
    step = {"n": 0}

    def exchange(cur):
        if rank == leave_rank and step["n"] == leave_after:
            os._exit(0)  # between steps: nothing of this rank is in flight
        step["n"] += 1
        nxt = torch.empty_like(cur)
        reqs = [dist.isend(cur, (rank + 1) % world), dist.irecv(nxt, (rank - 1) % world)]

        def wait():
            for r in reqs:
                r.wait()
            return nxt

        return wait

    t0 = time.monotonic()
    try:
        run_ring(rank, world, kv, lambda *a: None, exchange)
        outcome = "completed"
    except Exception as e:  # the transport reports the missing peer
        outcome = "error:" + type(e).__name__
    with open(out_path + f".{rank}", "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.2f}\n")
    os._exit(0)  # the group cannot be torn down cleanly without the peer


@pytest.mark.parametrize("world,leave_rank,leave_after", [(3, 1, 1), (4, 2, 2)])
def test_ring_rank_leaving_between_steps_fails_cleanly(world, leave_rank, leave_after, tmp_path):
    """A rank that leaves the ring between steps: no survivor hangs, and the
    two ranks that exchange with it (a ring rank talks only to rank - 1 and
    rank + 1) see their next exchange end with an error within the process
    group's timeout.  Ranks further away may finish their own exchanges."""
    out = str(tmp_path / "leave")
    mp.start_processes(_leaving_worker,
                       args=(world, _free_port(), out, leave_rank, leave_after),
                       nprocs=world, join=True, start_method="spawn")
    neighbours = {(leave_rank - 1) % world, (leave_rank + 1) % world}
    for r in range(world):
        if r == leave_rank:
            continue
        outcome, secs = (tmp_path / f"leave.{r}").read_text().split()
        assert float(secs) < 30.0, (r, secs)
        if r in neighbours:
            assert outcome.startswith("error:"), (r, outcome)
