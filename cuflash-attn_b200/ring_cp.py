"""Ring context-parallel causal attention forward.

No counterpart in the reference library (single-device, no collectives).
The sequence of length N is cut into 2P chunks of C = N / (2P) tokens and
rank r of P holds chunks r and 2P-1-r ("zigzag"), which gives every rank the
same amount of causal work.  Each rank keeps its two query chunks and passes
its two K/V chunks around the ring: at step s it holds the K/V chunks of rank
(r - s) mod P.  For every (query chunk c_q, K/V chunk c_k) pair with
c_k <= c_q it runs the library's partial forward
(``cuflash_attention_forward_partial_*``, causal on global positions) and
folds the result into a running (O, L) with the log-sum-exp merge
(``cuflash_lse_merge_f32``).  The next step's K/V travel over NCCL
send/recv (``torch.distributed.batch_isend_irecv``) while the current step
computes; every remote chunk lands in local HBM before a kernel reads it.

On the CUDA path all visible pairs of one step run through
``cuflash_attention_forward_cp_step_*``: one persistent launch per group of
pairs with distinct query chunks (``distinct_q_groups``), with the
log-sum-exp merge done in the kernel's epilogue.

The backward (``RingAttention.backward``) walks the same ring.  dQ of the
rank's query chunks accumulates locally in fp32; the dK/dV contributions of
the K/V chunks held at step s belong to rank (r - s) and travel the ring in
fp32 with them: the step's kernel (``cuflash_attention_backward_cp_step_*``,
all of the step's pairs in one launch) adds them into a zeroed part buffer,
and a side stream adds that part into the accumulator received from rank
r - 1 (``cuflash_accumulate_f32``) and sends the sum to rank r + 1, while the
next step computes.  After the last step one more hop brings every
accumulator home (``dkv_hops``).

The schedule (``ring_steps`` / ``visible_pairs`` / ``distinct_q_groups``) is
backend-independent and is exercised on CPU with gloo in the tests.
"""

from __future__ import annotations

import os

from dataclasses import dataclass
from typing import Callable, List, Sequence, Tuple


def zigzag_chunks(rank: int, world: int) -> Tuple[int, int]:
    """Global chunk indices held by `rank` (out of 2*world chunks)."""
    return rank, 2 * world - 1 - rank


def kv_owner(rank: int, step: int, world: int) -> int:
    """Rank whose K/V chunks `rank` holds at ring step `step`."""
    return (rank - step) % world


def visible_pairs(q_chunks: Sequence[int], k_chunks: Sequence[int]) -> List[Tuple[int, int]]:
    """(local query slot, local K/V slot) pairs with any unmasked key."""
    return [(qi, ki) for qi, qc in enumerate(q_chunks) for ki, kc in enumerate(k_chunks)
            if kc <= qc]


@dataclass
class RingStep:
    step: int
    owner: int
    k_chunks: Tuple[int, int]
    pairs: List[Tuple[int, int]]


def ring_steps(rank: int, world: int) -> List[RingStep]:
    q_chunks = zigzag_chunks(rank, world)
    out = []
    for s in range(world):
        owner = kv_owner(rank, s, world)
        k_chunks = zigzag_chunks(owner, world)
        out.append(RingStep(s, owner, k_chunks, visible_pairs(q_chunks, k_chunks)))
    return out


def distinct_q_groups(pairs: Sequence[Tuple]) -> List[List[Tuple]]:
    """Splits a step's pairs (first element = query slot) into launch groups
    in which every query slot appears at most once, keeping the order of the
    pairs of each slot (the in-kernel merge updates each slot once per
    launch)."""
    groups: List[List[Tuple]] = []
    for p in pairs:
        for g in groups:
            if all(x[0] != p[0] for x in g):
                g.append(p)
                break
        else:
            groups.append([p])
    return groups


def run_ring(rank: int, world: int, chunk: int, kv_local, compute_pair: Callable,
             exchange: Callable):
    """Drives the ring.  `kv_local` is this rank's K/V payload (opaque to the
    schedule); `compute_pair(q_slot, q_chunk, kv, k_slot, k_chunk)` folds one
    partial result into the caller's accumulators; `exchange(kv)` starts
    sending `kv` to rank+1 and receiving rank-1's payload, returning a
    callable that waits and yields the received payload."""
    q_chunks = zigzag_chunks(rank, world)
    cur = kv_local
    for st in ring_steps(rank, world):
        pending = exchange(cur) if st.step + 1 < world else None
        for qi, ki in st.pairs:
            compute_pair(qi, q_chunks[qi], cur, ki, st.k_chunks[ki])
        if pending is not None:
            cur = pending()
    return q_chunks


def dkv_hops(rank: int, world: int) -> List[int]:
    """Owners of the dK/dV accumulators rank `rank` sends after each step
    (step s: the owner of the K/V it held, (rank - s) mod world); the
    accumulator sent after the last step arrives at its owner."""
    return [kv_owner(rank, s, world) for s in range(world)]


def run_ring_backward(rank: int, world: int, kv_local, compute_step: Callable,
                      exchange: Callable, new_acc: Callable, add: Callable):
    """Host-side schedule of the ring backward, independent of the backend.
    `compute_step(step, kv, acc)` adds the step's dK/dV contributions of the
    K/V chunks `kv` into `acc`; `exchange(payload)` sends to rank+1 and
    returns a callable yielding rank-1's payload; `new_acc()` makes a zero
    accumulator and `add(dst, src)` sums two.  Returns this rank's own final
    dK/dV accumulator."""
    cur = kv_local
    acc_in = None
    for st in ring_steps(rank, world):
        pending = exchange(cur) if st.step + 1 < world else None
        part = new_acc()
        compute_step(st, cur, part)
        if acc_in is not None:
            part = add(acc_in(), part)
        acc_in = exchange(part) if world > 1 else (lambda p=part: p)
        if pending is not None:
            cur = pending()
    return acc_in()


# ---------------------------------------------------------------------------
# CUDA / NCCL backend
# ---------------------------------------------------------------------------

class RingAttention:
    """Context-parallel causal forward over a torch.distributed NCCL group.

    Each rank passes its zigzag shard as four contiguous tensors
    [B, H, C, D] (query/key/value of its two chunks) and gets back its two
    output chunks and their log-sum-exp.
    """

    def __init__(self, lib, group=None):
        self.lib = lib
        self.group = group

    def forward(self, q_ab, k_ab, v_ab, scale: float):
        """Runs on the current CUDA stream (the stream NCCL's P2P operations
        are ordered against)."""
        import torch
        import torch.distributed as dist

        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        Qa = q_ab[0]
        B, H, C, D = Qa.shape
        dev = Qa.device
        stream = torch.cuda.current_stream(dev)
        Qs = torch.stack(list(q_ab)).contiguous()  # [2, B, H, C, D]
        O_acc = torch.zeros((2, B, H, C, D), device=dev, dtype=torch.float32)
        L_acc = torch.full((2, B, H, C), float("-inf"), device=dev, dtype=torch.float32)
        # K/V travel as one buffer [2 (k, v), 2 (chunks), B, H, C, D]
        kv = torch.stack([torch.stack(list(k_ab)), torch.stack(list(v_ab))]).contiguous()
        spare = torch.empty_like(kv)
        state = {"spare": spare}
        q_chunks = zigzag_chunks(rank, world)

        def exchange(cur):
            nxt = state["spare"]
            ops = [dist.P2POp(dist.isend, cur, (rank + 1) % world, self.group),
                   dist.P2POp(dist.irecv, nxt, (rank - 1) % world, self.group)]
            reqs = dist.batch_isend_irecv(ops)

            def wait():
                for r in reqs:
                    r.wait()
                state["spare"] = cur  # the buffer just sent is free next step
                return nxt

            return wait

        cur = kv
        # The step launches leave SMs free for the concurrent NCCL transfer
        # (CUFLASH_CP_RESERVE_SMS, 16 by default); a single rank has no
        # transfer, so it gives them to the kernels.
        saved = os.environ.get("CUFLASH_CP_RESERVE_SMS")
        if world == 1:
            os.environ["CUFLASH_CP_RESERVE_SMS"] = "0"
        try:
            for st in ring_steps(rank, world):
                pending = exchange(cur) if st.step + 1 < world else None
                pairs = [(qi, ki, q_chunks[qi] * C, st.k_chunks[ki] * C) for qi, ki in st.pairs]
                for group in distinct_q_groups(pairs):
                    self.lib.forward_cp_step(Qs, cur[0], cur[1], O_acc, L_acc, group,
                                             causal=True, scale=scale, stream=stream)
                if pending is not None:
                    cur = pending()
        finally:
            if world == 1:
                if saved is None:
                    os.environ.pop("CUFLASH_CP_RESERVE_SMS", None)
                else:
                    os.environ["CUFLASH_CP_RESERVE_SMS"] = saved
        out = []
        for qi in range(2):
            o = torch.empty((B, H, C, D), device=dev, dtype=Qa.dtype)
            self.lib.convert(O_acc[qi], o, stream=stream)
            out.append(o)
        return out, [L_acc[0], L_acc[1]]

    def backward(self, q_ab, k_ab, v_ab, o_ab, l_ab, do_ab, scale: float):
        """Ring backward of ``forward``: the same zigzag shard plus the
        forward's outputs o_ab (two chunks), their log-sum-exp l_ab (fp32
        [B, H, C] each) and the output gradients do_ab.  Returns
        (dq_ab, dk_ab, dv_ab), two chunks each, in the input dtype."""
        import torch
        import torch.distributed as dist

        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        Qa = q_ab[0]
        B, H, C, D = Qa.shape
        dev = Qa.device
        lib = self.lib
        stream = torch.cuda.current_stream(dev)
        Qs = torch.stack(list(q_ab)).contiguous()
        dOs = torch.stack(list(do_ab)).contiguous()
        Os = torch.stack(list(o_ab)).contiguous()
        Ls = torch.stack([x.float() for x in l_ab]).contiguous()
        ws = lib.backward_cp_workspace(Qs)
        lib.backward_cp_prepare(Os, dOs, Ls, ws, stream=stream)
        kv = torch.stack([torch.stack(list(k_ab)), torch.stack(list(v_ab))]).contiguous()
        spare = torch.empty_like(kv)
        q_chunks = zigzag_chunks(rank, world)
        shape = (2, 2, B, H, C, D)  # (dK, dV) x (K/V slot)
        # Accumulators travelling the ring (one being sent, one receiving) and
        # the steps' part buffers (one written by the step kernel, one being
        # added on the side stream); the step kernel and the adds clear them.
        accs = [torch.zeros(shape, device=dev, dtype=torch.float32) for _ in range(2)]
        parts = ([torch.zeros(shape, device=dev, dtype=torch.float32) for _ in range(2)]
                 if world > 1 else [])
        side = torch.cuda.Stream(dev) if world > 1 else None
        part_free = [None, None]  # side-stream event: part buffer cleared
        state = {"spare": spare}

        def exchange_kv(cur):
            nxt = state["spare"]
            ops = [dist.P2POp(dist.isend, cur, (rank + 1) % world, self.group),
                   dist.P2POp(dist.irecv, nxt, (rank - 1) % world, self.group)]
            reqs = dist.batch_isend_irecv(ops)

            def wait():
                for r in reqs:
                    r.wait()
                state["spare"] = cur
                return nxt

            return wait

        saved = os.environ.get("CUFLASH_CP_RESERVE_SMS")
        if world == 1:
            os.environ["CUFLASH_CP_RESERVE_SMS"] = "0"
        cur = kv
        acc_reqs = None  # requests of the previous accumulator exchange
        acc_cur = 0      # index of the accumulator this rank adds into next
        try:
            for st in ring_steps(rank, world):
                pending = exchange_kv(cur) if st.step + 1 < world else None
                pairs = [(qi, ki, q_chunks[qi] * C, st.k_chunks[ki] * C) for qi, ki in st.pairs]
                if st.step == 0:
                    target = accs[0]
                else:
                    target = parts[st.step % 2]
                    ev = part_free[st.step % 2]
                    if ev is not None:
                        stream.wait_event(ev)
                if pairs:
                    lib.backward_cp_step(Qs, dOs, cur[0], cur[1], ws, target[0], target[1],
                                         pairs, causal=True, scale=scale, stream=stream)
                if world > 1:
                    done = torch.cuda.Event()
                    done.record(stream)
                    with torch.cuda.stream(side):
                        side.wait_event(done)
                        if st.step > 0:
                            for r in acc_reqs:
                                r.wait()  # the accumulator of this owner has arrived
                            lib.accumulate(accs[acc_cur], target, zero_src=True, stream=side)
                            freed = torch.cuda.Event()
                            freed.record(side)
                            part_free[st.step % 2] = freed
                        send, recv = accs[acc_cur], accs[1 - acc_cur]
                        ops = [dist.P2POp(dist.isend, send, (rank + 1) % world, self.group),
                               dist.P2POp(dist.irecv, recv, (rank - 1) % world, self.group)]
                        acc_reqs = dist.batch_isend_irecv(ops)
                        acc_cur = 1 - acc_cur
                if pending is not None:
                    cur = pending()
            if world > 1:
                for r in acc_reqs:
                    r.wait()  # on the compute stream: this rank's own accumulator
                stream.wait_stream(side)
        finally:
            if world == 1:
                if saved is None:
                    os.environ.pop("CUFLASH_CP_RESERVE_SMS", None)
                else:
                    os.environ["CUFLASH_CP_RESERVE_SMS"] = saved
        final = accs[acc_cur] if world > 1 else accs[0]
        dQs = torch.empty_like(Qs)
        lib.backward_cp_finish(ws, dQs, scale=scale, stream=stream)
        dk = torch.empty((2, B, H, C, D), device=dev, dtype=Qa.dtype)
        dv = torch.empty_like(dk)
        lib.convert(final[0], dk, stream=stream)
        lib.convert(final[1], dv, stream=stream)
        return [dQs[0], dQs[1]], [dk[0], dk[1]], [dv[0], dv[1]]
