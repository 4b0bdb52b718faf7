"""Test-side ring drivers for context parallelism.

They walk the library's own schedule (``ring_cp.ring_steps``, i.e.
``cuflash_cp_ring_schedule`` in libcuflash_attn_cp.so) in the order the C
ring driver does, with a pluggable transport and compute, so the tests can
run the ring over gloo with the fp64 oracle as the compute (CPU) or emulate
P ranks on one GPU.  The product ring is the C entry point
``cuflash_attention_{forward,backward}_cp_*``.
"""

from typing import Callable

import ring_cp


def run_ring(rank: int, world: int, kv_local, compute_pair: Callable, exchange: Callable,
             causal: bool = True):
    """Forward ring.  `kv_local` is this rank's K/V payload (opaque here);
    `compute_pair(q_slot, q_chunk, kv, k_slot, k_chunk)` folds one partial
    result into the caller's accumulators; `exchange(kv)` starts sending `kv`
    to rank+1 and receiving rank-1's payload, returning a callable that waits
    and yields the received payload."""
    q_chunks = ring_cp.zigzag_chunks(rank, world)
    cur = kv_local
    for st in ring_cp.ring_steps(rank, world, causal):
        pending = exchange(cur) if st.step + 1 < world else None
        for launch in st.launches:
            for qi, ki in launch:
                compute_pair(qi, q_chunks[qi], cur, ki, st.k_chunks[ki])
        if pending is not None:
            cur = pending()
    return q_chunks


def run_ring_backward(rank: int, world: int, kv_local, compute_step: Callable,
                      exchange: Callable, new_acc: Callable, add: Callable,
                      causal: bool = True):
    """Backward ring.  `compute_step(step, kv, acc)` adds the step's dK/dV
    contributions of the K/V chunks `kv` into `acc`; `exchange(payload)` sends
    to rank+1 and returns a callable yielding rank-1's payload; `new_acc()`
    makes a zero accumulator and `add(dst, src)` sums two.  The accumulator
    of each step travels to rank+1 after the step (as in the C driver), so the
    one received after the last step is this rank's own; it is returned."""
    cur = kv_local
    acc_in = None
    for st in ring_cp.ring_steps(rank, world, causal):
        pending = exchange(cur) if st.step + 1 < world else None
        part = new_acc()
        compute_step(st, cur, part)
        if acc_in is not None:
            part = add(acc_in(), part)
        acc_in = exchange(part) if world > 1 else (lambda p=part: p)
        if pending is not None:
            cur = pending()
    return acc_in()
