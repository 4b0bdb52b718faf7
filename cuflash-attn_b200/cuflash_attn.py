"""ctypes binding of the cuflash B200 library (host-side mirror of the
reference's Python interface).

The reference ships a ctypes wrapper (``examples/python_binding.py:51-170``:
``load_library`` / ``CuFlashAttn.forward`` / ``backward`` / ``check_error``)
and its integration test binds the same C ABI
(``tests/integration/test_pytorch_comparison.py:37-148``, library override
through the ``CUFLASH_LIB`` environment variable, ``:158-180``).  This module
keeps those names, argument meanings and error behaviour, binds every
``extern "C"`` entry point of ``include/cuflash/flash_attention.h`` and takes
torch CUDA tensors (torch is used for device memory and streams only; all
arithmetic happens in the library's CUDA kernels).

There is no fallback: if ``libcuflash_attn.so`` is missing or a call fails,
an exception is raised.
"""

from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path
from typing import Optional, Tuple

_HERE = Path(__file__).resolve().parent
DEFAULT_LIB = _HERE / "lib" / "libcuflash_attn.so"

SUCCESS = 0
INVALID_DIMENSION = 1
DIMENSION_MISMATCH = 2
NULL_POINTER = 3
CUDA_ERROR = 4
OUT_OF_MEMORY = 5
UNSUPPORTED_HEAD_DIM = 6
UNSUPPORTED_DTYPE = 7

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_B = ctypes.c_bool
_LL = ctypes.c_longlong

# name -> argtypes; every function returns int unless listed in _RESTYPES.
SIGNATURES = {
    "cuflash_attention_forward_f32": [_P] * 5 + [_I] * 4 + [_F, _B, _P],
    "cuflash_attention_forward_f16": [_P] * 5 + [_I] * 4 + [_F, _B, _P],
    "cuflash_attention_forward_bf16": [_P] * 5 + [_I] * 4 + [_F, _B, _P],
    "cuflash_attention_backward_f32": [_P] * 9 + [_I] * 4 + [_F, _B, _P],
    "cuflash_attention_backward_f16": [_P] * 9 + [_I] * 4 + [_F, _B, _P],
    "cuflash_attention_backward_bf16": [_P] * 9 + [_I] * 4 + [_F, _B, _P],
    "cuflash_error_string": [_I],
    "cuflash_attention_decode_f16": [_P] * 5 + [_I] * 4 + [_F, _I, _P],
    "cuflash_attention_decode_bf16": [_P] * 5 + [_I] * 4 + [_F, _I, _P],
    "cuflash_attention_decode_bf16_noalloc": [_P] * 5 + [_I] * 4 + [_F, _I, _P],
    "cuflash_attention_forward_partial_bf16": [_P] * 5 + [_I] * 5 + [_F, _LL, _LL, _B, _P],
    "cuflash_attention_forward_partial_f16": [_P] * 5 + [_I] * 5 + [_F, _LL, _LL, _B, _P],
    "cuflash_attention_decode_gqa_bf16": [_P] * 5 + [_I] * 5 + [_F, _I, _P],
    "cuflash_attention_decode_gqa_f16": [_P] * 5 + [_I] * 5 + [_F, _I, _P],
    "cuflash_attention_decode_paged_bf16": [_P] * 7 + [_I] * 7 + [_F, _I, _P],
    "cuflash_attention_decode_paged_f16": [_P] * 7 + [_I] * 7 + [_F, _I, _P],
    "cuflash_attention_forward_gqa_bf16": [_P] * 5 + [_I] * 6 + [_F, _B, _P],
    "cuflash_attention_forward_gqa_f16": [_P] * 5 + [_I] * 6 + [_F, _B, _P],
    "cuflash_attention_backward_gqa_bf16": [_P] * 9 + [_I] * 6 + [_F, _B, _P],
    "cuflash_attention_backward_gqa_f16": [_P] * 9 + [_I] * 6 + [_F, _B, _P],
    "cuflash_attention_forward_cp_step_bf16": [_P] * 5 + [_I] * 6 + [_F, _B, _I] + [_P] * 4
    + [_I, _P],
    "cuflash_attention_forward_cp_step_f16": [_P] * 5 + [_I] * 6 + [_F, _B, _I] + [_P] * 4
    + [_I, _P],
    "cuflash_attention_backward_cp_workspace_size": [_I] * 5,
    "cuflash_attention_backward_cp_prepare_bf16": [_P] * 4 + [_I] * 5 + [_P],
    "cuflash_attention_backward_cp_prepare_f16": [_P] * 4 + [_I] * 5 + [_P],
    "cuflash_attention_backward_cp_step_bf16": [_P] * 7 + [_I] * 6 + [_F, _B, _I] + [_P] * 4
    + [_I, _P],
    "cuflash_attention_backward_cp_step_f16": [_P] * 7 + [_I] * 6 + [_F, _B, _I] + [_P] * 4
    + [_I, _P],
    "cuflash_attention_backward_cp_finish_bf16": [_P] * 2 + [_I] * 5 + [_F, _P],
    "cuflash_attention_backward_cp_finish_f16": [_P] * 2 + [_I] * 5 + [_F, _P],
    "cuflash_accumulate_f32": [_P, _P, _LL, _B, _P],
    "cuflash_lse_merge_f32": [_P] * 4 + [_LL, _I, _P],
    "cuflash_convert_f32_to_bf16": [_P, _P, _LL, _P],
    "cuflash_convert_f32_to_f16": [_P, _P, _LL, _P],
    "cuflash_device_status": [],
    "cuflash_set_option": [ctypes.c_char_p, _I],
    "cuflash_profile_main_kernels": [_I],
    "cuflash_profile_read_ms": [_P, _I],
}
_RESTYPES = {"cuflash_error_string": ctypes.c_char_p,
             "cuflash_attention_backward_cp_workspace_size": ctypes.c_longlong}


def library_path(lib_path: Optional[str] = None) -> str:
    """Explicit argument, then ``CUFLASH_LIB``, then the in-tree build."""
    if lib_path:
        return str(lib_path)
    env = os.environ.get("CUFLASH_LIB")
    if env:
        return env
    return str(DEFAULT_LIB)


# The entry points the reference library exports (flash_attention.h:81-118).
REFERENCE_ABI = tuple(f"cuflash_attention_{pass_}_{sfx}" for pass_ in ("forward", "backward")
                      for sfx in ("f32", "f16", "bf16")) + ("cuflash_error_string",)


def load_library(lib_path: Optional[str] = None, reference_abi_only: bool = False) -> ctypes.CDLL:
    """Loads the library (RTLD_LOCAL) and declares every C-ABI signature.

    ``reference_abi_only`` binds only the reference's six entry points and
    ``cuflash_error_string``, so the same binding can drive a build of the
    reference library itself."""
    path = library_path(lib_path)
    if not Path(path).exists():
        raise RuntimeError(
            f"libcuflash_attn.so not found at {path}; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` or `make -C cuflash-attn_b200`"
        )
    lib = ctypes.CDLL(path, mode=os.RTLD_LOCAL)
    for name, argtypes in SIGNATURES.items():
        if reference_abi_only and name not in REFERENCE_ABI:
            continue
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    return lib


class CuFlashError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"CuFlash-Attn error {code}: {message}")
        self.code = code


_SUFFIX = {"float32": "f32", "float16": "f16", "bfloat16": "bf16"}


def _suffix(t) -> str:
    name = str(t.dtype).replace("torch.", "")
    if name not in _SUFFIX:
        raise CuFlashError(UNSUPPORTED_DTYPE, f"Unsupported data type {t.dtype}")
    return _SUFFIX[name]


def _ptr(t) -> ctypes.c_void_p:
    if t is None:
        return ctypes.c_void_p(0)
    if not t.is_cuda:
        raise ValueError("tensor must be on a CUDA device")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


def _stream_handle(stream) -> ctypes.c_void_p:
    if stream is None:
        import torch

        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


class CuFlashAttn:
    """Object interface over the C ABI (names follow the reference's
    ``examples/python_binding.py:CuFlashAttn``)."""

    def __init__(self, lib_path: Optional[str] = None, reference_abi_only: bool = False):
        self.lib = load_library(lib_path, reference_abi_only)

    def error_string(self, code: int) -> str:
        return self.lib.cuflash_error_string(int(code)).decode("utf-8")

    def check_error(self, code: int) -> None:
        if code != SUCCESS:
            raise CuFlashError(code, self.error_string(code))

    # -- reference surface -------------------------------------------------
    def forward(self, Q, K, V, causal: bool = False, scale: Optional[float] = None,
                O=None, L=None, stream=None) -> Tuple["torch.Tensor", "torch.Tensor"]:
        """O, L = attention(Q, K, V); Q/K/V [B,H,N,D] fp32/fp16/bf16."""
        import torch

        B, H, N, D = Q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        if O is None:
            O = torch.empty_like(Q)
        if L is None:
            L = torch.empty((B, H, N), device=Q.device, dtype=torch.float32)
        fn = getattr(self.lib, f"cuflash_attention_forward_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), B, H, N, D,
                            float(scale), bool(causal), _stream_handle(stream)))
        return O, L

    def backward(self, Q, K, V, O, L, dO, causal: bool = False, scale: Optional[float] = None,
                 dQ=None, dK=None, dV=None, stream=None):
        """dQ, dK, dV of attention given the forward's O and L."""
        import torch

        B, H, N, D = Q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        dQ = torch.empty_like(Q) if dQ is None else dQ
        dK = torch.empty_like(K) if dK is None else dK
        dV = torch.empty_like(V) if dV is None else dV
        fn = getattr(self.lib, f"cuflash_attention_backward_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), _ptr(dO), _ptr(dQ),
                            _ptr(dK), _ptr(dV), B, H, N, D, float(scale), bool(causal),
                            _stream_handle(stream)))
        return dQ, dK, dV

    # -- additive entry points ----------------------------------------------
    def decode(self, q, K, V, scale: Optional[float] = None, num_splits: int = 0,
               O=None, L=None, stream=None):
        """Split-KV decode: q [B,H,1,D] against K/V [B,H,Nkv,D]."""
        import torch

        B, H, Nkv, D = K.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(q) if O is None else O
        L = torch.empty((B, H), device=q.device, dtype=torch.float32) if L is None else L
        fn = getattr(self.lib, f"cuflash_attention_decode_{_suffix(q)}")
        self.check_error(fn(_ptr(q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), B, H, Nkv, D,
                            float(scale), int(num_splits), _stream_handle(stream)))
        return O, L

    def forward_partial(self, Q, K, V, q_offset: int, k_offset: int, causal: bool = True,
                        scale: Optional[float] = None, O=None, L=None, stream=None):
        """Normalised fp32 partial (O, L) of Q against one K/V chunk."""
        import torch

        B, H, Nq, D = Q.shape
        Nk = K.shape[2]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        O = torch.empty((B, H, Nq, D), device=Q.device, dtype=torch.float32) if O is None else O
        L = torch.empty((B, H, Nq), device=Q.device, dtype=torch.float32) if L is None else L
        fn = getattr(self.lib, f"cuflash_attention_forward_partial_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), B, H, Nq, Nk, D,
                            float(scale), int(q_offset), int(k_offset), bool(causal),
                            _stream_handle(stream)))
        return O, L

    def decode_gqa(self, q, K, V, scale: Optional[float] = None, num_splits: int = 0, O=None,
                   L=None, stream=None):
        """q [B,Hq,1,D] against a contiguous cache K/V [B,Hkv,Nkv,D]."""
        import torch

        B, Hq, _, D = q.shape
        Hkv, Nkv = K.shape[1], K.shape[2]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(q) if O is None else O
        L = torch.empty((B, Hq), device=q.device, dtype=torch.float32) if L is None else L
        fn = getattr(self.lib, f"cuflash_attention_decode_gqa_{_suffix(q)}")
        self.check_error(fn(_ptr(q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), B, Hq, Hkv, Nkv, D,
                            float(scale), int(num_splits), _stream_handle(stream)))
        return O, L

    def decode_paged(self, q, K_cache, V_cache, block_table, seq_lens,
                     scale: Optional[float] = None, num_splits: int = 0, O=None, L=None,
                     stream=None):
        """q [B,Hq,1,D] against a paged cache K/V [pages, page_size, Hkv, D]
        with block_table int32 [B, max_pages] and seq_lens int32 [B]."""
        import torch

        B, Hq, _, D = q.shape
        num_pages, page_size, Hkv, _ = K_cache.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(q) if O is None else O
        L = torch.empty((B, Hq), device=q.device, dtype=torch.float32) if L is None else L
        fn = getattr(self.lib, f"cuflash_attention_decode_paged_{_suffix(q)}")
        self.check_error(fn(_ptr(q), _ptr(K_cache), _ptr(V_cache), _ptr(block_table),
                            _ptr(seq_lens), _ptr(O), _ptr(L), B, Hq, Hkv, D, page_size,
                            block_table.shape[1], num_pages, float(scale), int(num_splits),
                            _stream_handle(stream)))
        return O, L

    def forward_gqa(self, Q, K, V, causal: bool = False, scale: Optional[float] = None, O=None,
                    L=None, stream=None):
        """Grouped-query forward: Q [B,Hq,Nq,D], K/V [B,Hkv,Nk,D]; causal is
        aligned bottom-right."""
        import torch

        B, Hq, Nq, D = Q.shape
        Hkv, Nk = K.shape[1], K.shape[2]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(Q) if O is None else O
        L = torch.empty((B, Hq, Nq), device=Q.device, dtype=torch.float32) if L is None else L
        fn = getattr(self.lib, f"cuflash_attention_forward_gqa_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), B, Hq, Hkv, Nq, Nk, D,
                            float(scale), bool(causal), _stream_handle(stream)))
        return O, L

    def backward_gqa(self, Q, K, V, O, L, dO, causal: bool = False,
                     scale: Optional[float] = None, dQ=None, dK=None, dV=None, stream=None):
        import torch

        B, Hq, Nq, D = Q.shape
        Hkv, Nk = K.shape[1], K.shape[2]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        dQ = torch.empty_like(Q) if dQ is None else dQ
        dK = torch.empty_like(K) if dK is None else dK
        dV = torch.empty_like(V) if dV is None else dV
        fn = getattr(self.lib, f"cuflash_attention_backward_gqa_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), _ptr(L), _ptr(dO), _ptr(dQ),
                            _ptr(dK), _ptr(dV), B, Hq, Hkv, Nq, Nk, D, float(scale),
                            bool(causal), _stream_handle(stream)))
        return dQ, dK, dV

    def forward_cp_step(self, Q, K, V, O_acc, L_acc, pairs, causal: bool = True,
                        scale: Optional[float] = None, reserve_sms: int = 0,
                        stream=None) -> None:
        """One context-parallel ring step in one launch.  Q [nq,B,H,C,D] and
        K, V [nk,B,H,C,D] hold stacked chunks; O_acc fp32 [nq,B,H,C,D] and
        L_acc fp32 [nq,B,H,C] are updated in place.  `pairs` lists up to four
        (q_slot, kv_slot, q_offset, kv_offset) with distinct q_slot;
        `reserve_sms` SMs stay free for concurrent transfers."""
        nq, B, H, C, D = Q.shape
        nk = K.shape[0]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        n = len(pairs)
        qs = (ctypes.c_int * max(n, 1))(*[int(x[0]) for x in pairs])
        ks = (ctypes.c_int * max(n, 1))(*[int(x[1]) for x in pairs])
        qo = (ctypes.c_longlong * max(n, 1))(*[int(x[2]) for x in pairs])
        ko = (ctypes.c_longlong * max(n, 1))(*[int(x[3]) for x in pairs])
        fn = getattr(self.lib, f"cuflash_attention_forward_cp_step_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(K), _ptr(V), _ptr(O_acc), _ptr(L_acc), nq, nk, B, H, C,
                            D, float(scale), bool(causal), n, ctypes.cast(qs, _P),
                            ctypes.cast(ks, _P), ctypes.cast(qo, _P), ctypes.cast(ko, _P),
                            int(reserve_sms), _stream_handle(stream)))

    @staticmethod
    def _pair_arrays(pairs):
        n = len(pairs)
        qs = (ctypes.c_int * max(n, 1))(*[int(x[0]) for x in pairs])
        ks = (ctypes.c_int * max(n, 1))(*[int(x[1]) for x in pairs])
        qo = (ctypes.c_longlong * max(n, 1))(*[int(x[2]) for x in pairs])
        ko = (ctypes.c_longlong * max(n, 1))(*[int(x[3]) for x in pairs])
        return n, qs, ks, qo, ko

    def backward_cp_workspace(self, Q):
        """A byte workspace for the context-parallel backward of the stacked
        query slots Q [nq,B,H,C,D] (kept across the ring steps)."""
        import torch

        nq, B, H, C, D = Q.shape
        nbytes = int(self.lib.cuflash_attention_backward_cp_workspace_size(nq, B, H, C, D))
        if nbytes <= 0:
            raise CuFlashError(INVALID_DIMENSION, self.error_string(INVALID_DIMENSION))
        return torch.empty(nbytes, dtype=torch.uint8, device=Q.device)

    def backward_cp_prepare(self, O, dO, L, workspace, stream=None) -> None:
        """O, dO [nq,B,H,C,D] (the forward's final output), L fp32 [nq,B,H,C]."""
        nq, B, H, C, D = O.shape
        fn = getattr(self.lib, f"cuflash_attention_backward_cp_prepare_{_suffix(O)}")
        self.check_error(fn(_ptr(O), _ptr(dO), _ptr(L), _ptr(workspace), nq, B, H, C, D,
                            _stream_handle(stream)))

    def backward_cp_step(self, Q, dO, K, V, workspace, dK_acc, dV_acc, pairs,
                         causal: bool = True, scale: Optional[float] = None,
                         reserve_sms: int = 0, stream=None) -> None:
        """One ring step of the context-parallel backward in one launch: Q, dO
        [nq,B,H,C,D], K, V [nk,B,H,C,D]; scale*dK and dV of the step are added
        into dK_acc / dV_acc fp32 [nk,B,H,C,D], dQ into the workspace.
        `pairs` lists up to four (q_slot, kv_slot, q_offset, kv_offset)."""
        nq, B, H, C, D = Q.shape
        nk = K.shape[0]
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        n, qs, ks, qo, ko = self._pair_arrays(pairs)
        fn = getattr(self.lib, f"cuflash_attention_backward_cp_step_{_suffix(Q)}")
        self.check_error(fn(_ptr(Q), _ptr(dO), _ptr(K), _ptr(V), _ptr(workspace), _ptr(dK_acc),
                            _ptr(dV_acc), nq, nk, B, H, C, D, float(scale), bool(causal), n,
                            ctypes.cast(qs, _P), ctypes.cast(ks, _P), ctypes.cast(qo, _P),
                            ctypes.cast(ko, _P), int(reserve_sms), _stream_handle(stream)))

    def backward_cp_finish(self, workspace, dQ, scale: Optional[float] = None,
                           stream=None) -> None:
        """dQ [nq,B,H,C,D] = scale * the accumulated dQ."""
        nq, B, H, C, D = dQ.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        fn = getattr(self.lib, f"cuflash_attention_backward_cp_finish_{_suffix(dQ)}")
        self.check_error(fn(_ptr(workspace), _ptr(dQ), nq, B, H, C, D, float(scale),
                            _stream_handle(stream)))

    def accumulate(self, dst, src, zero_src: bool = False, stream=None) -> None:
        """dst += src (fp32, same size); zero_src also clears src."""
        self.check_error(self.lib.cuflash_accumulate_f32(_ptr(dst), _ptr(src), dst.numel(),
                                                         bool(zero_src), _stream_handle(stream)))

    def lse_merge(self, O_acc, L_acc, O_part, L_part, stream=None) -> None:
        rows = L_acc.numel()
        D = O_acc.shape[-1]
        self.check_error(self.lib.cuflash_lse_merge_f32(_ptr(O_acc), _ptr(L_acc), _ptr(O_part),
                                                        _ptr(L_part), rows, D,
                                                        _stream_handle(stream)))

    def convert(self, src_f32, dst, stream=None) -> None:
        fn = getattr(self.lib, f"cuflash_convert_f32_to_{_suffix(dst)}")
        self.check_error(fn(_ptr(src_f32), _ptr(dst), src_f32.numel(), _stream_handle(stream)))

    def device_status(self) -> int:
        return int(self.lib.cuflash_device_status())

    def profile_main_kernels(self, num_launches: int) -> None:
        """Times the next `num_launches` backward main kernels (see
        cuflash_profile_main_kernels); 0 stops."""
        self.check_error(self.lib.cuflash_profile_main_kernels(int(num_launches)))

    def profile_read_ms(self, max_launches: int):
        """Durations (ms) of the profiled backward main kernels so far."""
        buf = (ctypes.c_float * max(int(max_launches), 1))()
        n = int(self.lib.cuflash_profile_read_ms(ctypes.cast(buf, _P), int(max_launches)))
        if n < 0:
            self.check_error(-n)
        return [float(buf[i]) for i in range(n)]

    def set_option(self, name: str, value: int) -> None:
        """Sets a process-wide option (see ``cuflash_set_option``); a
        negative value restores the built-in default."""
        self.check_error(self.lib.cuflash_set_option(name.encode(), int(value)))
