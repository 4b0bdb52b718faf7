"""Context-parallel backward on the GPU (cuflash_attention_backward_cp_*).

* P ranks emulated in one process on one GPU: every rank's ring steps run
  through the single-launch step entry, each step's dK/dV added straight into
  the owner's fp32 accumulator (the ring's travel is exercised on CPU with
  gloo and, with two GPUs, over NCCL below).  The assembled dQ/dK/dV must
  match the fp64 oracle's full causal backward within 2e-2 (the reference
  tests' fp16/bf16 bar) and the single-GPU backward of this library.
* One launch over several pairs equals one launch per pair.
* Pairs whose K/V blocks are partly invisible (K/V chunk starting inside or
  after the query chunk) match the oracle's per-pair backward.
* The ring entry point itself (cuflash_attention_backward_cp_*, NCCL) is
  tested in test_gpu_ring_cp_nccl.py.
"""

import numpy as np
import pytest

import oracle
import ring_cp
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _tdt(dt):
    import torch

    return torch.bfloat16 if dt == "bf16" else torch.float16


def _emulated_ring_backward(lib, Q, K, V, O, L, dO, world, C, scale):
    """Runs every rank's steps on this GPU; returns full-sequence dQ, dK, dV."""
    import torch

    B, H, N, D = Q.shape
    sl = lambda x, c: x[:, :, c * C:(c + 1) * C]
    stack = lambda x, cs: torch.stack([sl(x, c) for c in cs]).contiguous()
    dQ = torch.empty_like(Q)
    # fp32 dK/dV accumulator of every owner's two chunks
    acc = {o: torch.zeros((2, 2, B, H, C, D), device="cuda") for o in range(world)}
    for r in range(world):
        chunks = ring_cp.zigzag_chunks(r, world)
        Qs, dOs, Os = stack(Q, chunks), stack(dO, chunks), stack(O, chunks)
        Ls = stack(L, chunks)
        ws = lib.backward_cp_workspace(Qs)
        lib.backward_cp_prepare(Os, dOs, Ls, ws)
        for st in ring_cp.ring_steps(r, world):
            Ks, Vs = stack(K, st.k_chunks), stack(V, st.k_chunks)
            pairs = [(qi, ki, chunks[qi] * C, st.k_chunks[ki] * C) for qi, ki in st.pairs]
            a = acc[st.owner]
            lib.backward_cp_step(Qs, dOs, Ks, Vs, ws, a[0], a[1], pairs, causal=True,
                                 scale=scale)
        dQs = torch.empty_like(Qs)
        lib.backward_cp_finish(ws, dQs, scale=scale)
        for qi, c in enumerate(chunks):
            dQ[:, :, c * C:(c + 1) * C] = dQs[qi]
    dK = torch.empty_like(K)
    dV = torch.empty_like(V)
    for o in range(world):
        for ki, c in enumerate(ring_cp.zigzag_chunks(o, world)):
            dK[:, :, c * C:(c + 1) * C] = acc[o][0, ki].to(K.dtype)
            dV[:, :, c * C:(c + 1) * C] = acc[o][1, ki].to(V.dtype)
    return dQ, dK, dV


@pytest.mark.parametrize("world,C,D,dt", [
    (1, 256, 128, "bf16"),
    (2, 256, 128, "bf16"),
    (4, 128, 64, "bf16"),
    (2, 200, 128, "f16"),   # chunk not a multiple of the 128-row block
    (3, 96, 32, "bf16"),
    (8, 128, 64, "bf16"),   # the BASELINE CP world size
])
def test_cp_backward_emulated_ring_vs_fp64(lib, cuda, world, C, D, dt):
    import torch

    B, H = 1, 4
    N = 2 * world * C
    scale = 1.0 / np.sqrt(D)
    Qh, Kh, Vh, dOh = (round_to(oracle.normal((B, H, N, D), s), dt) for s in (51, 52, 53, 54))
    Q, K, V, dO = (to_dev(x, dt) for x in (Qh, Kh, Vh, dOh))
    O, L = lib.forward(Q, K, V, causal=True, scale=scale)
    dQ, dK, dV = _emulated_ring_backward(lib, Q, K, V, O, L, dO, world, C, scale)
    rQ, rK, rV = lib.backward(Q, K, V, O, L, dO, causal=True, scale=scale)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    gQ, gK, gV = oracle.backward_f64(Qh, Kh, Vh, dOh, scale, True)
    for got, ref in ((dQ, gQ), (dK, gK), (dV, gV)):
        assert max_err(host(got), ref) < TOL
    # and against the single-GPU backward: only accumulation order differs
    for got, ref in ((dQ, rQ), (dK, rK), (dV, rV)):
        assert max_err(host(got), host(ref)) < TOL


@pytest.mark.parametrize("D", [64, 128])
def test_cp_step_multi_pair_equals_single_pairs(lib, cuda, D):
    import torch

    B, H, C = 1, 4, 320
    g = torch.Generator(device="cuda").manual_seed(9)
    mk = lambda n: torch.randn((n, B, H, C, D), device="cuda", generator=g).to(torch.bfloat16)
    Q, dO, O = mk(2), mk(2), mk(2)
    K, V = mk(2), mk(2)
    L = (torch.randn((2, B, H, C), device="cuda", generator=g) + 8.0).contiguous()
    scale = 1.0 / np.sqrt(D)
    # a diagonal pair, two fully visible pairs sharing K/V slot 0, one sharing query slot 1
    pairs = [(0, 0, 3 * C, 3 * C), (1, 0, 5 * C, 3 * C), (1, 1, 5 * C, 4 * C),
             (0, 1, 7 * C, 4 * C)]
    outs = []
    for split in (False, True):
        ws = lib.backward_cp_workspace(Q)
        lib.backward_cp_prepare(O, dO, L, ws)
        dk = torch.zeros((2, B, H, C, D), device="cuda")
        dv = torch.zeros_like(dk)
        groups = [[p] for p in pairs] if split else [pairs]
        for grp in groups:
            lib.backward_cp_step(Q, dO, K, V, ws, dk, dv, grp, causal=True, scale=scale)
        # the fp32 dQ accumulator heads the workspace
        dq_acc = ws.view(torch.float32)[:Q.numel()].clone()
        outs.append((dq_acc, dk, dv))
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for a, b in zip(*outs):
        assert torch.allclose(a, b, rtol=1e-3, atol=1e-3), float((a - b).abs().max())


@pytest.mark.parametrize("rel", [-160, 64, 0, 1000])
def test_cp_step_partial_visibility_vs_pair_oracle(lib, cuda, rel):
    """Query chunk at global offset kv_offset + rel: with rel < 0 the K/V
    blocks past the queries' last position see no query and are skipped."""
    import torch

    B, H, C, D = 1, 2, 384, 64
    scale = 1.0 / np.sqrt(D)
    k_off = 512
    q_off = k_off + rel
    Qh, Kh, Vh, dOh, Oh = (round_to(oracle.normal((1, B, H, C, D), s), "bf16")
                           for s in (61, 62, 63, 64, 65))
    Lh = (oracle.normal((1, B, H, C), 66) * 0.5 + 6.0).astype(np.float32)
    Q, K, V, dO, O = (to_dev(x, "bf16") for x in (Qh, Kh, Vh, dOh, Oh))
    L = torch.from_numpy(Lh).cuda()
    ws = lib.backward_cp_workspace(Q)
    lib.backward_cp_prepare(O, dO, L, ws)
    dk = torch.zeros((1, B, H, C, D), device="cuda")
    dv = torch.zeros_like(dk)
    lib.backward_cp_step(Q, dO, K, V, ws, dk, dv, [(0, 0, q_off, k_off)], causal=True,
                         scale=scale)
    dq = torch.empty_like(Q)
    lib.backward_cp_finish(ws, dq, scale=scale)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    Dv = (dOh[0].astype(np.float64) * Oh[0]).sum(-1)
    gQ, gK, gV = oracle.backward_pair_f64(Qh[0], Kh[0], Vh[0], dOh[0], Lh[0], Dv, scale, True,
                                          q_off, k_off)
    for got, ref in ((dq[0], gQ), (dk[0], gK), (dv[0], gV)):
        # relative to the gradients' size, which is small with these statistics
        assert max_err(host(got), ref) < 1e-2 * float(np.abs(ref).max()) + 1e-4
    if rel < 0:  # K/V rows after the last query stay untouched
        last_key = C + rel  # keys 0..C+rel-1 are visible to some query
        assert float(dk[0, :, :, last_key:].abs().max()) == 0.0
