"""TEST INFRASTRUCTURE ONLY — numpy/ctypes front end of the CPU oracle
(``oracle/cpu_ref.cpp``), the restatement of the reference's CPU attention
(``tests/unit/test_forward.cu:21-118``, ``tests/unit/test_backward.cu:21-127``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module, always as the checker or the timed CPU
baseline, never as the product path.

Parity status: pinned.  ``tests/test_oracle.py`` checks the fp32 path
against golden vectors produced by the reference's own CUDA library
(``tests/golden/``) and against the reference tests' known-answer
identities.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_build" / "liboracle.so"
REF_LIB_PATH = _HERE / "_ref" / "libcuflash_attn_ref.so"

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_LL = ctypes.c_longlong
_I = ctypes.c_int

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL)
        L.oracle_fill_interleaved_uniform.argtypes = [ctypes.c_void_p] * 4 + [
            _LL, ctypes.c_uint, ctypes.c_float, ctypes.c_float]
        L.oracle_fill_uniform.argtypes = [_f32p, _LL, ctypes.c_uint, ctypes.c_float, ctypes.c_float]
        L.oracle_fill_normal.argtypes = [_f32p, _LL, ctypes.c_uint, ctypes.c_float, ctypes.c_float]
        L.oracle_forward_f32.argtypes = [_f32p, _f32p, _f32p, ctypes.c_void_p, ctypes.c_void_p,
                                         _LL, _LL, _I, _I, ctypes.c_float, _I, _I]
        L.oracle_backward_f32.argtypes = [_f32p] * 7 + [_LL, _LL, _I, _I, ctypes.c_float, _I, _I]
        L.oracle_forward_f64.argtypes = [_f32p, _f32p, _f32p, ctypes.c_void_p, ctypes.c_void_p,
                                         _LL, _LL, _I, _I, _I, ctypes.c_double, _I, _LL, _LL, _I]
        L.oracle_backward_f64.argtypes = [_f32p] * 4 + [_f64p] * 3 + [
            _LL, _LL, _I, _I, ctypes.c_double, _I, _I]
        L.oracle_backward_gen_f64.argtypes = [_f32p] * 4 + [ctypes.c_void_p] * 3 + [
            _LL, _LL, _I, _I, _I, ctypes.c_double, _I, _LL, _LL, _I]
        L.oracle_train_step_rows_f32.argtypes = [_f32p] * 9 + [_LL, _LL, _I, _I, ctypes.c_float,
                                                   _I, _I, _I, _I]
        L.oracle_train_step_rows_f32.restype = ctypes.c_longlong
        L.oracle_forward_rows_f64.argtypes = [_f32p] * 3 + [ctypes.c_void_p] * 2 + [
            _LL, _LL, ctypes.c_void_p, _I, _I, _I, ctypes.c_double, _I, _I]
        for f in ("oracle_fill_interleaved_uniform", "oracle_fill_uniform", "oracle_fill_normal",
                  "oracle_forward_f32", "oracle_backward_f32", "oracle_forward_f64",
                  "oracle_backward_f64", "oracle_backward_gen_f64", "oracle_forward_rows_f64"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def _vp(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---- generators -------------------------------------------------------------

def interleaved_uniform(shape, seed, lo, hi, count=3):
    """The reference tests' fill: mt19937(seed), uniform_real_distribution
    <float>(lo, hi), tensors interleaved per index (test_forward.cu:133-139)."""
    n = int(np.prod(shape))
    arrs = [np.empty(n, np.float32) for _ in range(count)]
    d = arrs[3] if count == 4 else None
    lib().oracle_fill_interleaved_uniform(_vp(arrs[0]), _vp(arrs[1]), _vp(arrs[2]), _vp(d), n,
                                          seed, lo, hi)
    return [a.reshape(shape) for a in arrs]


def uniform(shape, seed, lo=-1.0, hi=1.0):
    a = np.empty(int(np.prod(shape)), np.float32)
    lib().oracle_fill_uniform(a, a.size, seed, lo, hi)
    return a.reshape(shape)


def normal(shape, seed, std=1.0):
    a = np.empty(int(np.prod(shape)), np.float32)
    lib().oracle_fill_normal(a, a.size, seed, 0.0, std)
    return a.reshape(shape)


# ---- reference CPU path (fp32) --------------------------------------------------

def forward_f32(Q, K, V, scale, causal, units=None, nthreads=1, want_o=True, want_l=True):
    """Reference fp32 CPU forward over (b,h) units [u0,u1) of [B,H,N,D]."""
    Q, K, V = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V))
    B, H, N, D = Q.shape
    u0, u1 = units if units is not None else (0, B * H)
    O = np.zeros_like(Q) if want_o else None
    L = np.zeros((B, H, N), np.float32) if want_l else None
    lib().oracle_forward_f32(Q, K, V, _vp(O), _vp(L), u0, u1, N, D, float(scale), int(causal),
                             int(nthreads))
    return O, L


def backward_f32(Q, K, V, dO, scale, causal, units=None, nthreads=1):
    Q, K, V, dO = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V, dO))
    B, H, N, D = Q.shape
    u0, u1 = units if units is not None else (0, B * H)
    dQ, dK, dV = (np.zeros_like(Q) for _ in range(3))
    lib().oracle_backward_f32(Q, K, V, dO, dQ, dK, dV, u0, u1, N, D, float(scale), int(causal),
                              int(nthreads))
    return dQ, dK, dV


def train_step_rows_f32(Q, K, V, dO, scale, causal, units, row_begin, row_step, nthreads):
    """One fwd+bwd step of the reference CPU path over units [u0,u1) of
    [U,N,D] arrays, sampled rows only; returns visible (i,j) pairs processed.
    Used to time the reference CPU path on a bounded sample."""
    U, N, D = Q.shape
    O = np.zeros_like(Q)
    L = np.zeros((U, N), np.float32)
    dQ, dK, dV = (np.zeros_like(Q) for _ in range(3))
    return lib().oracle_train_step_rows_f32(Q, K, V, dO, O, L, dQ, dK, dV, units[0], units[1], N,
                                            D, float(scale), int(causal), int(row_begin),
                                            int(row_step), int(nthreads))


# ---- fp64 ground truth -------------------------------------------------------------

def forward_f64(Q, K, V, scale, causal, q_offset=0, k_offset=0, units=None, nthreads=8):
    """fp64 forward; Q [B,H,Nq,D], K/V [B,H,Nk,D]; causal mask on global
    positions (key k_offset+j hidden from query q_offset+i iff j' > i')."""
    Q, K, V = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V))
    B, H, Nq, D = Q.shape
    Nk = K.shape[2]
    u0, u1 = units if units is not None else (0, B * H)
    O = np.zeros((B, H, Nq, D), np.float64)
    L = np.zeros((B, H, Nq), np.float64)
    lib().oracle_forward_f64(Q, K, V, _vp(O), _vp(L), u0, u1, Nq, Nk, D, float(scale),
                             int(causal), int(q_offset), int(k_offset), int(nthreads))
    return O, L


def forward_rows_f64(Q, K, V, scale, causal, rows, nthreads=16):
    """fp64 forward of the query rows `rows` only; Q, K, V [B,H,N,D], row
    index = global position.  Returns O [B,H,len(rows),D], L [B,H,len(rows)]."""
    Q, K, V = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V))
    B, H, N, D = Q.shape
    r = np.ascontiguousarray(rows, np.int64)
    O = np.zeros((B, H, len(r), D), np.float64)
    L = np.zeros((B, H, len(r)), np.float64)
    lib().oracle_forward_rows_f64(Q, K, V, _vp(O), _vp(L), 0, B * H, _vp(r), len(r), N, D,
                                  float(scale), int(causal), int(nthreads))
    return O, L


def backward_f64(Q, K, V, dO, scale, causal, units=None, nthreads=8):
    Q, K, V, dO = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V, dO))
    B, H, N, D = Q.shape
    u0, u1 = units if units is not None else (0, B * H)
    dQ, dK, dV = (np.zeros(Q.shape, np.float64) for _ in range(3))
    lib().oracle_backward_f64(Q, K, V, dO, dQ, dK, dV, u0, u1, N, D, float(scale), int(causal),
                              int(nthreads))
    return dQ, dK, dV


def backward_gen_f64(Q, K, V, dO, scale, causal, q_offset=0, k_offset=0, units=None,
                     nthreads=8):
    """fp64 backward with separate lengths: Q, dO [B,H,Nq,D], K/V [B,H,Nk,D],
    causal on global positions (key k_offset+j hidden from query q_offset+i
    iff k_offset+j > q_offset+i)."""
    Q, K, V, dO = (np.ascontiguousarray(x, np.float32) for x in (Q, K, V, dO))
    B, H, Nq, D = Q.shape
    Nk = K.shape[2]
    u0, u1 = units if units is not None else (0, B * H)
    dQ = np.zeros(Q.shape, np.float64)
    dK, dV = (np.zeros(K.shape, np.float64) for _ in range(2))
    lib().oracle_backward_gen_f64(Q, K, V, dO, _vp(dQ), _vp(dK), _vp(dV), u0, u1, Nq, Nk, D,
                                  float(scale), int(causal), int(q_offset), int(k_offset),
                                  int(nthreads))
    return dQ, dK, dV


def backward_pair_f64(Q, K, V, dO, L, Dv, scale, causal, q_offset=0, k_offset=0):
    """Contribution of one (query chunk, key chunk) pair to dQ, dK, dV, given
    the statistics of the whole softmax row: L the natural-log LSE over every
    key of the sequence, Dv = rowsum(dO * O) with the final output O.  Same
    per-element algebra as the reference's CPU backward
    (tests/unit/test_backward.cu:21-127: P = softmax row, dP = dO V^T,
    dS = P (dP - D), dQ = scale dS K, dK = scale dS^T Q, dV = P^T dO), with P
    taken as exp(scale q.k - L) so that the pairs of a sequence sum to the
    full backward.  Causal on global positions (key k_offset+j hidden from
    query q_offset+i iff k_offset+j > q_offset+i).  numpy fp64, [B,H,N,D]."""
    Q, K, V, dO = (np.asarray(x, np.float64) for x in (Q, K, V, dO))
    L = np.asarray(L, np.float64)
    Dv = np.asarray(Dv, np.float64)
    Nq, Nk = Q.shape[2], K.shape[2]
    S = scale * np.einsum("bhid,bhjd->bhij", Q, K)
    fin = np.isfinite(L)[..., None]
    P = np.where(fin, np.exp(S - np.where(fin, L[..., None], 0.0)), 0.0)
    if causal:
        qpos = q_offset + np.arange(Nq)[:, None]
        kpos = k_offset + np.arange(Nk)[None, :]
        P = np.where(kpos > qpos, 0.0, P)
    dV = np.einsum("bhij,bhid->bhjd", P, dO)
    dP = np.einsum("bhid,bhjd->bhij", dO, V)
    dS = P * (dP - Dv[..., None])
    dQ = scale * np.einsum("bhij,bhjd->bhid", dS, K)
    dK = scale * np.einsum("bhij,bhid->bhjd", dS, Q)
    return dQ, dK, dV


def gqa_forward_f64(Q, K, V, scale, causal):
    """Grouped-query forward: Q [B,Hq,Nq,D], K/V [B,Hkv,Nk,D], query head h
    reads K/V head h // (Hq/Hkv); causal is bottom-right aligned (query i sees
    key j iff j <= i + Nk - Nq)."""
    g = Q.shape[1] // K.shape[1]
    Kr, Vr = np.repeat(K, g, axis=1), np.repeat(V, g, axis=1)
    return forward_f64(Q, Kr, Vr, scale, causal, q_offset=K.shape[2] - Q.shape[2], k_offset=0)


def gqa_backward_f64(Q, K, V, dO, scale, causal):
    """Grouped-query backward (same conventions); dK/dV of a K/V head sum its
    query heads' contributions."""
    B, Hq, Nq, D = Q.shape
    Hkv, Nk = K.shape[1], K.shape[2]
    g = Hq // Hkv
    Kr, Vr = np.repeat(K, g, axis=1), np.repeat(V, g, axis=1)
    qo = Nk - Nq
    # q_offset may be negative (more queries than keys): shift both sides
    dQ, dK, dV = backward_gen_f64(Q, Kr, Vr, dO, scale, causal, q_offset=max(qo, 0),
                                  k_offset=max(-qo, 0))
    dK = dK.reshape(B, Hkv, g, Nk, D).sum(axis=2)
    dV = dV.reshape(B, Hkv, g, Nk, D).sum(axis=2)
    return dQ, dK, dV


def decode_f64(q, K, V, scale):
    """q [B,H,1,D], K/V [B,H,Nkv,D] -> O [B,H,1,D], L [B,H] (fp64)."""
    O, L = forward_f64(q, K, V, scale, causal=False)
    return O, L[..., 0]


# ---- dtype rounding helpers (round to nearest even, as __float2bfloat16_rn) ------

def round_bf16(x):
    """float32 -> nearest bfloat16 value, returned as float32."""
    a = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((a >> 16) & 1) + np.uint32(0x7FFF)
    out = ((a + r) & np.uint32(0xFFFF0000)).view(np.float32)
    nan = np.isnan(np.asarray(x, np.float32))
    return np.where(nan, np.float32(np.nan), out).astype(np.float32)


def round_f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
