"""The context-parallel ring entry points of libcuflash_attn_cp.so
(cuflash_attention_{forward,backward}_cp_*, NCCL), called through the C ABI.

* One rank (world = 1, no communicator): the ring's single step on the
  caller's stream, against the single-GPU entry points on the whole sequence
  and the fp64 oracle.
* Two GPUs, and every GPU of the box when it has more: one process per GPU,
  an NCCL communicator made through the library's helpers (its unique id
  handed out over a gloo group), the same full-sequence inputs on every rank;
  each rank's output chunks and gradients against the single-GPU entry points
  and the fp64 oracle on sampled rows, over both transports (copy engine
  over CUDA IPC, NCCL send/recv).  Three shapes in a row: the second reuses
  the copy-engine context of the first, the third needs larger buffers and
  rebuilds it.  NVLS is off (NCCL_NVLS_ENABLE=0).
* A rank whose export never gets signalled (a host-side test switch): the
  other rank's bounded wait gives up, its transport status reads 1, and the
  next call returns CUDA_ERROR on both ranks until the status is cleared.
"""

import os
import socket

import numpy as np
import pytest

import oracle
import ring_cp
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the reference tests' fp16/bf16 bar


def _chunks(x, chunks, C):
    return [x[:, :, c * C:(c + 1) * C].contiguous() for c in chunks]


def _check_rank(lib, ring, rank, world, Qh, Kh, Vh, dOh, dt, causal, C):
    """Runs the ring forward and backward for `rank` and returns the largest
    errors against the single-GPU library and fp64 (sampled rows)."""
    import torch

    Q, K, V, dO = (to_dev(x, dt) for x in (Qh, Kh, Vh, dOh))
    D = Q.shape[-1]
    scale = 1.0 / np.sqrt(D)
    O, L = lib.forward(Q, K, V, causal=causal, scale=scale)
    rQ, rK, rV = lib.backward(Q, K, V, O, L, dO, causal=causal, scale=scale)
    chunks = ring_cp.zigzag_chunks(rank, world)
    cs = lambda x: _chunks(x, chunks, C)
    outs, lses = ring.forward(cs(Q), cs(K), cs(V), scale, causal=causal)
    dq, dk, dv = ring.backward(cs(Q), cs(K), cs(V), outs, lses, cs(dO), scale, causal=causal)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    err_lib = 0.0
    err_64 = 0.0
    for i, c in enumerate(chunks):
        s = slice(c * C, (c + 1) * C)
        pairs = ((outs[i], O[:, :, s]), (lses[i], L[:, :, s]), (dq[i], rQ[:, :, s]),
                 (dk[i], rK[:, :, s]), (dv[i], rV[:, :, s]))
        err_lib = max([err_lib] + [max_err(host(a), host(b)) for a, b in pairs])
        rows = np.arange(c * C, (c + 1) * C, 5)
        O64, L64 = oracle.forward_rows_f64(Qh, Kh, Vh, scale, causal, rows)
        err_64 = max(err_64, max_err(host(outs[i])[:, :, rows - c * C], O64),
                     max_err(host(lses[i])[:, :, rows - c * C], L64))
    return err_lib, err_64


@pytest.mark.parametrize("dt,causal,C,D", [("bf16", True, 384, 128), ("f16", True, 200, 64),
                                           ("bf16", False, 256, 128)])
def test_ring_entry_single_rank(lib, cuda, dt, causal, C, D):
    B, H = 1, 4
    N = 2 * C
    arrs = [round_to(oracle.normal((B, H, N, D), s), dt) for s in (61, 62, 63, 64)]
    err_lib, err_64 = _check_rank(lib, ring_cp.RingAttention(), 0, 1, *arrs, dt, causal, C)
    assert err_lib < TOL and err_64 < TOL
    # the gradients also against fp64 (whole sequence: one rank holds it all)
    import torch

    Q, K, V, dO = (to_dev(x, dt) for x in arrs)
    scale = 1.0 / np.sqrt(D)
    ring = ring_cp.RingAttention()
    outs, lses = ring.forward(_chunks(Q, (0, 1), C), _chunks(K, (0, 1), C),
                              _chunks(V, (0, 1), C), scale, causal=causal)
    dq, dk, dv = ring.backward(_chunks(Q, (0, 1), C), _chunks(K, (0, 1), C),
                               _chunks(V, (0, 1), C), outs, lses, _chunks(dO, (0, 1), C), scale,
                               causal=causal)
    torch.cuda.synchronize()
    gQ, gK, gV = oracle.backward_f64(*arrs, scale, causal)
    for c in range(2):
        s = slice(c * C, (c + 1) * C)
        assert max_err(host(dq[c]), gQ[:, :, s]) < TOL
        assert max_err(host(dk[c]), gK[:, :, s]) < TOL
        assert max_err(host(dv[c]), gV[:, :, s]) < TOL


def test_ring_entry_rejects_a_mismatched_communicator(lib, cuda):
    """A one-rank communicator passed with world = 1 but rank 0 works; the
    entry checks that comm's size and rank match world and rank."""
    import torch

    uid = ring_cp.nccl_unique_id()
    comm = ring_cp.NcclComm(1, 0, uid)
    try:
        B, H, C, D = 1, 2, 128, 64
        x = torch.zeros((2, B, H, C, D), device="cuda", dtype=torch.bfloat16)
        O = torch.empty_like(x)
        L = torch.empty((2, B, H, C), device="cuda")
        fn = ring_cp.load_cp_library().cuflash_attention_forward_cp_bf16
        p = lambda t: ring_cp.cf._ptr(t)
        st = ring_cp.cf._stream_handle(None)
        # comm has one rank: world 2 (with a matching sequence length) is a mismatch
        assert fn(p(x), p(x), p(x), p(O), p(L), B, H, 4 * C, D, 0.1, True, comm.handle, 0, 2,
                  -1, st) == ring_cp.cf.DIMENSION_MISMATCH
        assert fn(p(x), p(x), p(x), p(O), p(L), B, H, 2 * C, D, 0.1, True, comm.handle, 0, 1,
                  -1, st) == ring_cp.cf.SUCCESS
        torch.cuda.synchronize()
    finally:
        comm.destroy()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, result_dir, transport):
    import torch
    import torch.distributed as dist

    import cuflash_attn

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta

    # gloo only hands out the NCCL unique id; the ring's traffic is NCCL's
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    comm = None
    try:
        obj = [ring_cp.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = ring_cp.NcclComm(world, rank, obj[0])
        lib = cuflash_attn.CuFlashAttn()
        ring_cp.set_transport(transport)
        ring = ring_cp.RingAttention(comm)
        B, H, D = 1, 4, 128
        lines = []
        for dt, causal, seed, C in (("bf16", True, 17, 256), ("f16", False, 23, 256),
                                    ("bf16", True, 29, 384)):
            N = 2 * world * C
            arrs = [round_to(oracle.normal((B, H, N, D), seed + i), dt) for i in range(4)]
            err_lib, err_64 = _check_rank(lib, ring, rank, world, *arrs, dt, causal, C)
            lines.append(f"{dt} {causal} {err_lib} {err_64} {err_lib < TOL and err_64 < TOL}")
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write("\n".join(lines) + "\n")
    finally:
        dist.barrier()
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


def _run_ring(world, tmp_path, transport):
    import torch.multiprocessing as mp

    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path), transport),
                       nprocs=world, join=True, start_method="spawn")
    for r in range(world):
        for line in (tmp_path / f"rank{r}.txt").read_text().split("\n"):
            if line:
                assert line.split()[-1] == "True", (r, line)


@pytest.mark.parametrize("transport", [ring_cp.TRANSPORT_PEER, ring_cp.TRANSPORT_NCCL])
def test_ring_entry_over_nccl_two_gpus(tmp_path, transport):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_ring(2, tmp_path, transport)


@pytest.mark.parametrize("transport", [ring_cp.TRANSPORT_PEER, ring_cp.TRANSPORT_NCCL])
def test_ring_entry_over_nccl_every_gpu(tmp_path, transport):
    """The same over every GPU of the box when it has more than two (eight
    on the BASELINE's context-parallel setting), one rank per GPU."""
    import torch

    world = torch.cuda.device_count()
    if world <= 2:
        pytest.skip("needs more than two GPUs")
    _run_ring(world, tmp_path, transport)


def _timeout_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["CUFLASH_CP_WAIT_LIMIT_MS"] = "300"
    if rank == 1:
        os.environ["CUFLASH_CP_TEST_SKIP_EXPORT_SIGNAL"] = "1"
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    comm = None
    try:
        obj = [ring_cp.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = ring_cp.NcclComm(world, rank, obj[0])
        ring_cp.set_transport(ring_cp.TRANSPORT_PEER)
        fn = ring_cp.load_cp_library().cuflash_attention_forward_cp_bf16
        B, H, C, D = 1, 2, 128, 64
        x = torch.randn((2, B, H, C, D), device="cuda").to(torch.bfloat16)
        O = torch.empty_like(x)
        L = torch.empty((2, B, H, C), device="cuda")
        p = ring_cp.cf._ptr
        st = ring_cp.cf._stream_handle(None)
        call = lambda: fn(p(x), p(x), p(x), p(O), p(L), B, H, 2 * world * C, D, 0.1, True,
                          comm.handle, rank, world, -1, st)
        codes = [call()]  # rank 0's wait for rank 1's export gives up after 300 ms
        torch.cuda.synchronize()
        codes.append(call())  # refused on both ranks: rank 0's status is set
        status = ring_cp.transport_status() if rank == 0 else 0
        dist.barrier()
        codes.append(call())  # accepted again once the status has been read
        torch.cuda.synchronize()
        ring_cp.transport_status()
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{codes[0]} {codes[1]} {codes[2]} {status}\n")
    finally:
        dist.barrier()
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


def test_peer_transport_wait_gives_up(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_timeout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    r0 = (tmp_path / "rank0.txt").read_text().split()
    r1 = (tmp_path / "rank1.txt").read_text().split()
    ok, err = str(ring_cp.cf.SUCCESS), str(ring_cp.cf.CUDA_ERROR)
    assert r0[:3] == [ok, err, ok] and r1[:3] == [ok, err, ok], (r0, r1)
    assert r0[3] == "1"
