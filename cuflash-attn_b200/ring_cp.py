"""Context-parallel causal attention: ctypes binding of
``libcuflash_attn_cp.so``.

No counterpart in the reference library (single-device, no collectives).
The ring runs in the C library (``cuflash_attention_{forward,backward}_cp_*``,
``include/cuflash/flash_attention_cp.h``): the sequence of length N is cut
into 2P chunks of C = N / (2P) tokens, rank r of P holds chunks r and
2P-1-r ("zigzag", equal causal work per rank), keeps its query chunks and
at step s computes with the K/V chunks of rank r - s while the next ones
travel: by default pulled from that rank's CUDA-IPC-shared export with a
copy-engine copy (the backward pushes its fp32 dK/dV straight to the
owner), or passed around the ring with NCCL send/recv (the backward then
carries fp32 dK/dV accumulators with the K/V they belong to).  This module
only stacks torch tensors into the library's shard layout, creates NCCL
communicators through the library's helpers, selects the transport, and reads
the ring schedule (``cuflash_cp_ring_schedule``) for callers and tests that
drive the per-step entry points themselves.

There is no fallback: if the library is missing or a call fails, an
exception is raised.
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Tuple

import cuflash_attn as cf

_HERE = Path(__file__).resolve().parent
DEFAULT_CP_LIB = _HERE / "lib" / "libcuflash_attn_cp.so"
UNIQUE_ID_BYTES = 128  # NCCL_UNIQUE_ID_BYTES

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_B = ctypes.c_bool

CP_SIGNATURES = {
    "cuflash_attention_forward_cp_bf16": [_P] * 5 + [_I] * 4 + [_F, _B, _P, _I, _I, _I, _P],
    "cuflash_attention_forward_cp_f16": [_P] * 5 + [_I] * 4 + [_F, _B, _P, _I, _I, _I, _P],
    "cuflash_attention_backward_cp_bf16": [_P] * 9 + [_I] * 4 + [_F, _B, _P, _I, _I, _I, _P],
    "cuflash_attention_backward_cp_f16": [_P] * 9 + [_I] * 4 + [_F, _B, _P, _I, _I, _I, _P],
    "cuflash_cp_ring_schedule": [_I, _I, _I, _B] + [_P] * 7,
    "cuflash_cp_nccl_unique_id": [_P, _I],
    "cuflash_cp_nccl_comm_init": [_P, _I, _P, _I],
    "cuflash_cp_nccl_comm_init_config": [_P, _I, _P, _I, _I],
    "cuflash_cp_nccl_comm_destroy": [_P],
    "cuflash_cp_set_transport": [_I],
    "cuflash_cp_transport_status": [],
}

_cp_lib = None


def load_cp_library(lib_path: Optional[str] = None) -> ctypes.CDLL:
    """Loads libcuflash_attn_cp.so (it brings libcuflash_attn.so from its own
    directory and the process's libnccl.so.2) and declares its signatures."""
    global _cp_lib
    if lib_path is None and _cp_lib is not None:
        return _cp_lib
    path = str(lib_path or os.environ.get("CUFLASH_CP_LIB") or DEFAULT_CP_LIB)
    if not Path(path).exists():
        raise RuntimeError(f"libcuflash_attn_cp.so not found at {path}; build it with "
                           "`make -C cuflash-attn_b200`")
    lib = ctypes.CDLL(path, mode=os.RTLD_LOCAL)
    for name, argtypes in CP_SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    # from libcuflash_attn.so, which the CP library links
    lib.cuflash_error_string.argtypes = [_I]
    lib.cuflash_error_string.restype = ctypes.c_char_p
    if lib_path is None:
        _cp_lib = lib
    return lib


def _check(code: int) -> None:
    if code != cf.SUCCESS:
        msg = load_cp_library().cuflash_error_string(int(code)).decode("utf-8")
        raise cf.CuFlashError(code, msg)


# ---------------------------------------------------------------------------
# schedule
# ---------------------------------------------------------------------------

def zigzag_chunks(rank: int, world: int) -> Tuple[int, int]:
    """Global chunk indices held by `rank` (out of 2*world chunks)."""
    return rank, 2 * world - 1 - rank


def kv_owner(rank: int, step: int, world: int) -> int:
    """Rank whose K/V chunks `rank` holds at ring step `step`."""
    return (rank - step) % world


@dataclass
class RingStep:
    step: int
    owner: int
    k_chunks: Tuple[int, int]
    pairs: List[Tuple[int, int]]                       # (query slot, K/V slot)
    launches: List[List[Tuple[int, int]]] = field(default_factory=list)  # forward launches


def ring_schedule(rank: int, world: int, step: int, causal: bool = True) -> RingStep:
    """The library's schedule for one step (``cuflash_cp_ring_schedule``)."""
    lib = load_cp_library()
    owner, n = ctypes.c_int(), ctypes.c_int()
    arrs = [(ctypes.c_int * 4)() for _ in range(5)]
    _check(lib.cuflash_cp_ring_schedule(rank, world, step, bool(causal), ctypes.byref(owner),
                                        ctypes.byref(n), *[ctypes.cast(a, _P) for a in arrs]))
    qs, ks, qc, kc, ln = ([a[i] for i in range(n.value)] for a in arrs)
    pairs = list(zip(qs, ks))
    launches: List[List[Tuple[int, int]]] = [[] for _ in range(max(ln, default=-1) + 1)]
    for p, l in zip(pairs, ln):
        launches[l].append(p)
    return RingStep(step, owner.value, zigzag_chunks(owner.value, world), pairs, launches)


def ring_steps(rank: int, world: int, causal: bool = True) -> List[RingStep]:
    return [ring_schedule(rank, world, s, causal) for s in range(world)]


def dkv_hops(rank: int, world: int) -> List[int]:
    """Owners of the dK/dV accumulators rank `rank` sends after each step of
    the ring backward (step s: the owner of the K/V it held, (rank - s) mod
    world); the accumulator sent after the last step arrives at its owner."""
    return [kv_owner(rank, s, world) for s in range(world)]


# ---------------------------------------------------------------------------
# NCCL communicator and the ring entry points
# ---------------------------------------------------------------------------

def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (make it on one rank, give it to every rank)."""
    buf = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
    _check(load_cp_library().cuflash_cp_nccl_unique_id(ctypes.cast(buf, _P), UNIQUE_ID_BYTES))
    return buf.raw


TRANSPORT_PEER = 0  # copy engine over CUDA IPC (the library's default)
TRANSPORT_NCCL = 1  # NCCL send/recv ring


def set_transport(transport: int) -> None:
    """Transport of the ring entry points for this process
    (cuflash_cp_set_transport); every rank must choose the same."""
    _check(load_cp_library().cuflash_cp_set_transport(int(transport)))


def transport_status() -> int:
    """Reads and clears the copy-engine transport's status (1: a wait for
    another rank gave up)."""
    return int(load_cp_library().cuflash_cp_transport_status())


class NcclComm:
    """An NCCL communicator over `world` ranks on the current CUDA device
    (blocking, created through the library).  ``max_ctas`` > 0 caps the CTAs
    NCCL's kernels use (ncclConfig_t.maxCTAs); 0 keeps NCCL's default."""

    def __init__(self, world: int, rank: int, unique_id: bytes, max_ctas: int = 0):
        self.world, self.rank = world, rank
        self.handle = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, UNIQUE_ID_BYTES)
        _check(load_cp_library().cuflash_cp_nccl_comm_init_config(
            ctypes.byref(self.handle), world, ctypes.cast(buf, _P), rank, int(max_ctas)))

    def destroy(self) -> None:
        if self.handle:
            _check(load_cp_library().cuflash_cp_nccl_comm_destroy(self.handle))
            self.handle = ctypes.c_void_p()


class RingAttention:
    """Context-parallel causal attention of one rank's zigzag shard through
    the library's ring entry points (transport: :func:`set_transport`).
    ``comm`` is an :class:`NcclComm` (or None with a single rank).  Each rank
    passes its shard as two chunks [B, H, C, D] (global chunks rank and
    2*world-1-rank)."""

    def __init__(self, comm: Optional[NcclComm] = None, rank: int = 0, world: int = 1,
                 reserve_sms: int = -1):
        self.lib = load_cp_library()
        self.comm = comm
        self.rank = comm.rank if comm is not None else rank
        self.world = comm.world if comm is not None else world
        self.reserve_sms = reserve_sms

    def _comm(self):
        return self.comm.handle if self.comm is not None else ctypes.c_void_p(0)

    def forward(self, q_ab, k_ab, v_ab, scale: Optional[float] = None, causal: bool = True,
                stream=None):
        """Returns ([O_a, O_b], [L_a, L_b]) for the rank's two query chunks."""
        import torch

        Qs = torch.stack(list(q_ab)).contiguous()  # [2, B, H, C, D]
        Ks = torch.stack(list(k_ab)).contiguous()
        Vs = torch.stack(list(v_ab)).contiguous()
        _, B, H, C, D = Qs.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(Qs)
        L = torch.empty((2, B, H, C), device=Qs.device, dtype=torch.float32)
        fn = getattr(self.lib, f"cuflash_attention_forward_cp_{cf._suffix(Qs)}")
        _check(fn(cf._ptr(Qs), cf._ptr(Ks), cf._ptr(Vs), cf._ptr(O), cf._ptr(L), B, H,
                  2 * self.world * C, D, float(scale), bool(causal), self._comm(), self.rank,
                  self.world, int(self.reserve_sms), cf._stream_handle(stream)))
        return [O[0], O[1]], [L[0], L[1]]

    def backward(self, q_ab, k_ab, v_ab, o_ab, l_ab, do_ab, scale: Optional[float] = None,
                 causal: bool = True, stream=None):
        """Ring backward of ``forward``: the same shard plus the forward's
        outputs o_ab, their log-sum-exp l_ab (fp32 [B, H, C] each) and the
        output gradients do_ab.  Returns (dq_ab, dk_ab, dv_ab), two chunks each."""
        import torch

        Qs, Ks, Vs, Os, dOs = (torch.stack(list(x)).contiguous()
                               for x in (q_ab, k_ab, v_ab, o_ab, do_ab))
        Ls = torch.stack([x.float() for x in l_ab]).contiguous()
        _, B, H, C, D = Qs.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        dQ, dK, dV = torch.empty_like(Qs), torch.empty_like(Ks), torch.empty_like(Vs)
        fn = getattr(self.lib, f"cuflash_attention_backward_cp_{cf._suffix(Qs)}")
        _check(fn(cf._ptr(Qs), cf._ptr(Ks), cf._ptr(Vs), cf._ptr(Os), cf._ptr(Ls), cf._ptr(dOs),
                  cf._ptr(dQ), cf._ptr(dK), cf._ptr(dV), B, H, 2 * self.world * C, D,
                  float(scale), bool(causal), self._comm(), self.rank, self.world,
                  int(self.reserve_sms), cf._stream_handle(stream)))
        return [dQ[0], dQ[1]], [dK[0], dK[1]], [dV[0], dV[1]]
