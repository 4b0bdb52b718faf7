"""C-ABI boundary tests that need no GPU (the reference's host-only smoke
tests: tests/integration/test_api_smoke.cpp, tests/package_smoke/main.cpp,
and the validation half of tests/unit/test_error_handling.cu).

Argument validation runs before any CUDA call, so invalid calls return their
error code on a machine without a GPU.  Where the reference library was
built here (oracle/_ref), every invalid call is also made against it and the
two return codes must agree.
"""

import ctypes
import math
import re
from pathlib import Path

import pytest

import cuflash_attn as cf
import oracle

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "cuflash" / "flash_attention.h"

FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
NUL = ctypes.c_void_p(0)
STREAM = ctypes.c_void_p(0)


def declared_c_symbols():
    text = HEADER.read_text()
    c_part = text[text.index('extern "C"'):]
    return sorted(set(re.findall(r"CUFLASH_EXPORT\s+[\w\s\*]+?\b(cuflash_\w+)\s*\(", c_part)))


def test_header_declares_reference_abi():
    syms = declared_c_symbols()
    for name in cf.REFERENCE_ABI:
        assert name in syms
    assert set(syms) == set(cf.SIGNATURES), "binding and header disagree"


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(cf.library_path(), mode=ctypes.RTLD_LOCAL)
    for name in declared_c_symbols():
        assert hasattr(lib, name), name


CP_HEADER = ROOT / "include" / "cuflash" / "flash_attention_cp.h"


def test_cp_library_exports_every_declared_symbol():
    """libcuflash_attn_cp.so (the NCCL ring) exports exactly what
    flash_attention_cp.h declares, and the ctypes binding covers it."""
    import subprocess

    import ring_cp

    text = CP_HEADER.read_text()
    c_part = text[text.index('extern "C"'):]
    declared = set(re.findall(r"CUFLASH_EXPORT\s+[\w\s\*]+?\b(cuflash_\w+)\s*\(", c_part))
    assert declared == set(ring_cp.CP_SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", str(ring_cp.DEFAULT_CP_LIB)],
                         capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert exported == declared, exported ^ declared


def test_cp_comm_helpers_validate_before_nccl():
    """The communicator helpers reject bad arguments before any NCCL call
    (so these run without a GPU)."""
    import ctypes

    import ring_cp

    lib = ring_cp.load_cp_library()
    h = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(ring_cp.UNIQUE_ID_BYTES)
    P = ctypes.c_void_p
    assert lib.cuflash_cp_nccl_comm_init_config(None, 2, ctypes.cast(uid, P), 0, 0) == \
        cf.NULL_POINTER
    assert lib.cuflash_cp_nccl_comm_init_config(ctypes.byref(h), 2, None, 0, 0) == cf.NULL_POINTER
    for world, rank, ctas in ((0, 0, 0), (2, 2, 0), (2, -1, 0), (2, 0, -1)):
        assert lib.cuflash_cp_nccl_comm_init_config(ctypes.byref(h), world, ctypes.cast(uid, P),
                                                    rank, ctas) == cf.INVALID_DIMENSION
    assert lib.cuflash_cp_nccl_comm_init(ctypes.byref(h), 2, ctypes.cast(uid, P), 5) == \
        cf.INVALID_DIMENSION
    assert lib.cuflash_cp_nccl_unique_id(None, 128) == cf.NULL_POINTER
    assert lib.cuflash_cp_nccl_unique_id(ctypes.cast(uid, P), 4) == cf.INVALID_DIMENSION
    assert lib.cuflash_cp_nccl_comm_destroy(None) == cf.NULL_POINTER


def test_cp_transport_switch_and_status_need_no_gpu():
    """cuflash_cp_set_transport accepts 0 (copy engine) and 1 (NCCL) only;
    the transport status reads 0 before any wait ran."""
    import ring_cp

    lib = ring_cp.load_cp_library()
    assert lib.cuflash_cp_set_transport(2) == cf.INVALID_DIMENSION
    assert lib.cuflash_cp_set_transport(-1) == cf.INVALID_DIMENSION
    try:
        ring_cp.set_transport(ring_cp.TRANSPORT_NCCL)
        ring_cp.set_transport(ring_cp.TRANSPORT_PEER)
    finally:
        ring_cp.set_transport(ring_cp.TRANSPORT_PEER)
    assert ring_cp.transport_status() == 0


def test_library_hides_internal_symbols():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", cf.library_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    internal = [s for s in exported if "detail" in s or "fa_fwd_kernel" in s]
    assert not internal, internal


EXPECTED_STRINGS = {
    0: "Success",
    1: "Invalid dimension: dimensions must be positive",
    2: "Dimension mismatch: Q, K, V tensors have incompatible shapes",
    3: "Null pointer: input or output pointer is null",
    4: "CUDA error occurred",
    5: "Out of memory: insufficient GPU memory",
    6: "Unsupported head_dim: must be 32, 64, or 128",
    7: "Unsupported data type",
    99: "Unknown error",
}


def test_error_strings_byte_exact(lib):
    # tests/unit/test_error_handling.cu:236-254 pins these strings
    for code, s in EXPECTED_STRINGS.items():
        assert lib.error_string(code) == s


def _fwd(lib, sfx, q=FAKE, k=FAKE, v=FAKE, o=FAKE, l=FAKE, B=1, H=1, N=16, D=32, scale=0.125,
         causal=False):
    fn = getattr(lib.lib, f"cuflash_attention_forward_{sfx}")
    return fn(q, k, v, o, l, B, H, N, D, scale, causal, STREAM)


def _bwd(lib, sfx, ptrs=None, B=1, H=1, N=16, D=32, scale=0.125):
    p = [FAKE] * 9 if ptrs is None else ptrs
    fn = getattr(lib.lib, f"cuflash_attention_backward_{sfx}")
    return fn(*p, B, H, N, D, scale, False, STREAM)


INVALID_FWD = [
    # (kwargs, expected) — tests/unit/test_error_handling.cu:21-233
    (dict(q=NUL), 3), (dict(k=NUL), 3), (dict(v=NUL), 3), (dict(o=NUL), 3), (dict(l=NUL), 3),
    (dict(B=0), 1), (dict(B=-1), 1), (dict(H=0), 1), (dict(N=0), 1), (dict(D=0), 1),
    (dict(D=48), 6), (dict(D=256), 6), (dict(D=16), 6),
    (dict(scale=float("nan")), 1), (dict(scale=float("inf")), 1), (dict(scale=-1.0), 1),
    # order: null before dims, dims before head_dim, head_dim before scale
    (dict(q=NUL, B=0), 3), (dict(B=0, D=48), 1), (dict(D=48, scale=float("nan")), 6),
]


@pytest.mark.parametrize("sfx", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("kwargs,expected", INVALID_FWD)
def test_forward_validation(lib, sfx, kwargs, expected):
    assert _fwd(lib, sfx, **kwargs) == expected


@pytest.mark.parametrize("sfx", ["f32", "f16", "bf16"])
def test_backward_validation(lib, sfx):
    for idx in range(9):  # each of Q,K,V,O,L,dO,dQ,dK,dV null
        ptrs = [FAKE] * 9
        ptrs[idx] = NUL
        assert _bwd(lib, sfx, ptrs) == 3
    # gradient pointers are checked before the dimensions (:69-79)
    ptrs = [FAKE] * 9
    ptrs[6] = NUL
    assert _bwd(lib, sfx, ptrs, B=0) == 3
    assert _bwd(lib, sfx, B=0) == 1
    assert _bwd(lib, sfx, D=48) == 6
    assert _bwd(lib, sfx, scale=-0.5) == 1


@pytest.mark.parametrize("sfx", ["f32", "f16", "bf16"])
def test_validation_matches_reference_library(lib, ref_lib, sfx):
    for kwargs, expected in INVALID_FWD:
        assert _fwd(ref_lib, sfx, **kwargs) == _fwd(lib, sfx, **kwargs) == expected
    for B, D, scale in [(0, 32, 0.1), (1, 48, 0.1), (1, 32, math.nan), (2, 100, -1.0)]:
        assert _bwd(ref_lib, sfx, B=B, D=D, scale=scale) == _bwd(lib, sfx, B=B, D=D, scale=scale)
    for s in EXPECTED_STRINGS:
        assert ref_lib.error_string(s) == lib.error_string(s)


@pytest.mark.parametrize("sfx", ["f16", "bf16"])
def test_decode_validation(lib, sfx):
    fn = getattr(lib.lib, f"cuflash_attention_decode_{sfx}")
    args = lambda **kw: [kw.get(n, FAKE) for n in "qkvol"] + [
        kw.get("B", 1), kw.get("H", 1), kw.get("N", 64), kw.get("D", 64),
        kw.get("scale", 0.1), kw.get("splits", 0), STREAM]
    assert fn(*args(q=NUL)) == 3
    assert fn(*args(l=NUL)) == 3
    assert fn(*args(N=0)) == 1
    assert fn(*args(D=96)) == 6
    assert fn(*args(scale=float("nan"))) == 1
    assert fn(*args(splits=-1)) == 1
    assert fn(*args(splits=65)) == 1


@pytest.mark.parametrize("sfx", ["f16", "bf16"])
def test_partial_and_merge_validation(lib, sfx):
    fn = getattr(lib.lib, f"cuflash_attention_forward_partial_{sfx}")
    base = [FAKE] * 5 + [1, 1, 16, 16, 64, 0.1, 0, 0, True, STREAM]
    a = list(base)
    a[11] = -1
    assert fn(*a) == 1
    a = list(base)
    a[3] = NUL
    assert fn(*a) == 3
    a = list(base)
    a[9] = 80
    assert fn(*a) == 6
    m = lib.lib.cuflash_lse_merge_f32
    assert m(NUL, FAKE, FAKE, FAKE, 4, 64, STREAM) == 3
    assert m(FAKE, FAKE, FAKE, FAKE, 0, 64, STREAM) == 1
    assert m(FAKE, FAKE, FAKE, FAKE, 4, 0, STREAM) == 1


@pytest.mark.parametrize("sfx", ["f16", "bf16"])
def test_gqa_validation(lib, sfx):
    fwd = getattr(lib.lib, f"cuflash_attention_forward_gqa_{sfx}")
    bwd = getattr(lib.lib, f"cuflash_attention_backward_gqa_{sfx}")

    def f(B=1, Hq=8, Hkv=2, Nq=16, Nk=32, D=64, scale=0.1, nul=None):
        a = [FAKE] * 5 + [B, Hq, Hkv, Nq, Nk, D, scale, True, STREAM]
        if nul is not None:
            a[nul] = NUL
        return fwd(*a)

    def b(Hq=8, Hkv=2, nul=None):
        a = [FAKE] * 9 + [1, Hq, Hkv, 16, 32, 64, 0.1, True, STREAM]
        if nul is not None:
            a[nul] = NUL
        return bwd(*a)

    assert f(nul=2) == 3 and f(nul=4) == 3
    assert f(Nq=0) == 1 and f(Nk=-1) == 1 and f(Hkv=0) == 1
    assert f(Hq=6, Hkv=4) == 2                 # heads not divisible: DIMENSION_MISMATCH
    assert f(D=48) == 6
    assert f(scale=float("inf")) == 1 and f(scale=-1.0) == 1
    assert b(nul=5) == 3 and b(nul=8) == 3     # dO / dV checked like the reference
    assert b(Hq=9, Hkv=2) == 2


@pytest.mark.parametrize("sfx", ["f16", "bf16"])
def test_decode_gqa_paged_validation(lib, sfx):
    g = getattr(lib.lib, f"cuflash_attention_decode_gqa_{sfx}")
    pg = getattr(lib.lib, f"cuflash_attention_decode_paged_{sfx}")

    def cg(Hq=8, Hkv=2, N=64, D=128, splits=0, nul=None):
        a = [FAKE] * 5 + [1, Hq, Hkv, N, D, 0.1, splits, STREAM]
        if nul is not None:
            a[nul] = NUL
        return g(*a)

    def cp(Hq=8, Hkv=2, D=128, ps=16, mp=4, npg=8, splits=0, nul=None):
        a = [FAKE] * 7 + [1, Hq, Hkv, D, ps, mp, npg, 0.1, splits, STREAM]
        if nul is not None:
            a[nul] = NUL
        return pg(*a)

    assert cg(nul=1) == 3 and cg(N=0) == 1 and cg(Hq=6, Hkv=4) == 2 and cg(D=80) == 6
    assert cg(splits=65) == 1 and cg(splits=-1) == 1
    assert cp(nul=3) == 3 and cp(nul=4) == 3        # block table / seq_lens
    assert cp(ps=24) == 1 and cp(ps=0) == 1          # page size a power of two
    assert cp(mp=0) == 1 and cp(npg=0) == 1
    assert cp(Hq=9) == 2


@pytest.mark.parametrize("sfx", ["f16", "bf16"])
def test_cp_step_validation(lib, sfx):
    import ctypes

    fn = getattr(lib.lib, f"cuflash_attention_forward_cp_step_{sfx}")

    def arr(ct, vals):
        return ctypes.cast((ct * len(vals))(*vals), ctypes.c_void_p)

    def call(q=(0, 1), k=(0, 1), qo=(0, 64), ko=(0, 64), n=2, D=64, nq=2, nk=2, ptr=None,
             reserve=0):
        args = [FAKE] * 5 + [nq, nk, 1, 2, 64, D, 0.1, True, n, arr(ctypes.c_int, q),
                             arr(ctypes.c_int, k), arr(ctypes.c_longlong, qo),
                             arr(ctypes.c_longlong, ko), reserve, STREAM]
        if ptr is not None:
            args[ptr] = NUL
        return fn(*args)

    assert call(ptr=0) == 3                       # Q null
    assert call(ptr=4) == 3                       # L_acc null
    assert call(ptr=14) == 3                      # q_slot array null
    assert call(D=80) == 6
    assert call(n=0) == 1 and call(n=5) == 1      # 1..4 pairs
    assert call(q=(0, 0)) == 1                    # one launch merges each slot once
    assert call(q=(0, 2)) == 1                    # slot out of range
    assert call(k=(0, -1)) == 1
    assert call(qo=(0, -64)) == 1                 # negative global offset
    assert call(nq=0) == 1
    assert call(reserve=-1) == 1                  # SM reserve must be >= 0


@pytest.mark.parametrize("sfx", ["f16", "bf16"])
def test_cp_backward_validation(lib, sfx):
    import ctypes

    L = lib.lib
    assert L.cuflash_attention_backward_cp_workspace_size(2, 1, 2, 200, 64) == 4 * (
        2 * 2 * 200 * 64 + 2 * 2 * 2 * 256)
    assert L.cuflash_attention_backward_cp_workspace_size(2, 1, 2, 200, 80) == 0
    assert L.cuflash_attention_backward_cp_workspace_size(0, 1, 2, 200, 64) == 0

    prep = getattr(L, f"cuflash_attention_backward_cp_prepare_{sfx}")
    assert prep(NUL, FAKE, FAKE, FAKE, 2, 1, 2, 64, 64, STREAM) == 3
    assert prep(FAKE, FAKE, FAKE, NUL, 2, 1, 2, 64, 64, STREAM) == 3
    assert prep(FAKE, FAKE, FAKE, FAKE, 2, 1, 2, 64, 48, STREAM) == 6
    assert prep(FAKE, FAKE, FAKE, FAKE, 2, 0, 2, 64, 64, STREAM) == 1

    fin = getattr(L, f"cuflash_attention_backward_cp_finish_{sfx}")
    assert fin(NUL, FAKE, 2, 1, 2, 64, 64, 0.1, STREAM) == 3
    assert fin(FAKE, FAKE, 2, 1, 2, 64, 64, float("nan"), STREAM) == 1
    assert fin(FAKE, FAKE, 2, 1, 2, -1, 64, 0.1, STREAM) == 1

    fn = getattr(L, f"cuflash_attention_backward_cp_step_{sfx}")

    def arr(ct, vals):
        return ctypes.cast((ct * len(vals))(*vals), ctypes.c_void_p)

    def call(q=(0, 1), k=(0, 0), qo=(0, 64), ko=(0, 0), n=2, D=64, nq=2, nk=2, ptr=None,
             scale=0.1, reserve=0):
        args = [FAKE] * 7 + [nq, nk, 1, 2, 64, D, scale, True, n, arr(ctypes.c_int, q),
                             arr(ctypes.c_int, k), arr(ctypes.c_longlong, qo),
                             arr(ctypes.c_longlong, ko), reserve, STREAM]
        if ptr is not None:
            args[ptr] = NUL
        return fn(*args)

    assert call(ptr=0) == 3                       # Q null
    assert call(ptr=4) == 3                       # workspace null
    assert call(ptr=6) == 3                       # dV_acc null
    assert call(ptr=18) == 3                      # kv_slot array null
    assert call(D=96) == 6
    assert call(n=0) == 1 and call(n=5) == 1      # 1..4 pairs
    assert call(q=(0, 2)) == 1                    # query slot out of range
    assert call(k=(0, 2)) == 1                    # K/V slot out of range
    assert call(ko=(0, -1)) == 1                  # negative global offset
    assert call(nk=0) == 1
    assert call(scale=-1.0) == 1
    assert call(reserve=-2) == 1
    # a repeated (query slot, K/V slot) pair would add its gradients twice
    assert call(q=(1, 1), k=(0, 0), qo=(64, 64), ko=(0, 0)) == 1

    acc = L.cuflash_accumulate_f32
    assert acc(NUL, FAKE, 16, False, STREAM) == 3
    assert acc(FAKE, FAKE, 6, False, STREAM) == 1              # count a multiple of 4
    assert acc(ctypes.c_void_p(0x1004), FAKE, 16, False, STREAM) == 1  # 16-byte alignment


def test_oracle_is_test_infrastructure_only():
    """The product path must not import the oracle."""
    pkg = ROOT / "cuflash-attn_b200"
    for f in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cuh")):
        text = f.read_text()
        assert "import oracle" not in text and "liboracle" not in text, f
    assert "TEST INFRASTRUCTURE ONLY" in (ROOT / "oracle" / "cpu_ref.cpp").read_text()
    assert oracle.LIB_PATH.name == "liboracle.so"


def test_workspace_oom_fault_injection(lib):
    """Host-side fault injection: a failing workspace allocation surfaces as
    OUT_OF_MEMORY (the reference maps cudaMallocAsync failure the same way,
    src/backward/flash_attention_backward_typed.cu:378-387).  The request
    fails before any CUDA call, so no GPU is involved."""
    lib.set_option("CUFLASH_FAULT_WORKSPACE_OOM", 1)
    try:
        for sfx in ("f16", "bf16"):
            assert _bwd(lib, sfx, N=256, D=64) == cf.OUT_OF_MEMORY
            fn = getattr(lib.lib, f"cuflash_attention_decode_{sfx}")
            assert fn(FAKE, FAKE, FAKE, FAKE, FAKE, 2, 2, 4096, 128, 0.1, 8,
                      STREAM) == cf.OUT_OF_MEMORY
    finally:
        lib.set_option("CUFLASH_FAULT_WORKSPACE_OOM", -1)


def test_set_option_validation(lib):
    assert lib.lib.cuflash_set_option(None, 1) == cf.NULL_POINTER
    assert lib.lib.cuflash_set_option(b"CUFLASH_NO_SUCH_OPTION", 1) == cf.INVALID_DIMENSION
    assert lib.lib.cuflash_set_option(b"CUFLASH_RESERVE_SMS", -1) == cf.SUCCESS


def test_profile_hook_validation(lib):
    """The backward main-kernel profiling hook: argument checks and an empty
    read need no GPU (nothing is recorded until a backward runs)."""
    import ctypes

    assert lib.lib.cuflash_profile_main_kernels(-1) == cf.INVALID_DIMENSION
    assert lib.lib.cuflash_profile_main_kernels(0) == cf.SUCCESS
    assert lib.lib.cuflash_profile_read_ms(None, 4) == -cf.NULL_POINTER
    buf = (ctypes.c_float * 4)()
    assert lib.lib.cuflash_profile_read_ms(ctypes.cast(buf, ctypes.c_void_p), -1) == \
        -cf.INVALID_DIMENSION
    assert lib.profile_read_ms(4) == []
