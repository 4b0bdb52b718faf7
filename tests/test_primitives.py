"""The reference's primitive API (cuflash::kernels::matmul_* / online_softmax_*
/ tile_io, include/cuflash/kernels/*.cuh) on the C++ ABI, without a GPU: the
library exports every symbol the reference library exports (golden list
from the reference's own build, tests/golden/reference_symbols.txt), and
invalid calls return the reference's codes (validation precedes any CUDA
call; where oracle/_ref exists the reference library is called too, the
host-side half of tests/unit/test_{matmul,online_softmax,tile_io}.cu)."""

import ctypes
from pathlib import Path

import pytest

import cuflash_attn as cf
import oracle
from primitive_abi import MM_FORMS, MM_SHAPES, TILE_SHAPES, Primitives

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_symbols.txt"
FAKE = ctypes.c_void_p(0x1000)
NUL = ctypes.c_void_p(0)
STREAM = ctypes.c_void_p(0)


def _libs():
    libs = [Primitives(cf.library_path())]
    if oracle.REF_LIB_PATH.exists():
        libs.append(Primitives(oracle.REF_LIB_PATH))
    return libs


def test_exports_every_reference_symbol():
    import subprocess

    want = GOLDEN.read_text().split()
    assert len(want) == 75
    out = subprocess.run(["nm", "-D", "--defined-only", cf.library_path()], capture_output=True,
                         text=True, check=True).stdout
    have = {ln.split()[-1] for ln in out.splitlines() if len(ln.split()) == 3}
    missing = [s for s in want if s not in have]
    assert not missing, missing


def test_primitive_symbols_resolve():
    p = Primitives(cf.library_path())
    for form in MM_FORMS:
        for M, N, K in MM_SHAPES:
            p.matmul(form, M, N, K)
    for R, C in TILE_SHAPES:
        for half in (False, True):
            p.load_tile(R, C, half)
            p.store_tile(R, C, half)
    p.roundtrip()
    p.softmax_init(), p.softmax_update(), p.softmax_finalize(), p.softmax_forward()


@pytest.mark.parametrize("which", range(2))
def test_primitive_validation(which):
    libs = _libs()
    if which >= len(libs):
        pytest.skip("reference build oracle/_ref is absent")
    p = libs[which]
    for form in MM_FORMS:
        f = p.matmul(form, 64, 64, 32)
        assert f(NUL, FAKE, FAKE, 1.0, STREAM) == 3
        assert f(FAKE, NUL, FAKE, 1.0, STREAM) == 3
        assert f(FAKE, FAKE, NUL, 1.0, STREAM) == 3
    for half in (False, True):
        ld = p.load_tile(64, 64, half)
        assert ld(NUL, FAKE, 0, 0, 128, 128, 128, STREAM) == 3
        assert ld(FAKE, NUL, 0, 0, 128, 128, 128, STREAM) == 3
        assert ld(FAKE, FAKE, -1, 0, 128, 128, 128, STREAM) == 1     # start before the matrix
        assert ld(FAKE, FAKE, 128, 0, 128, 128, 128, STREAM) == 1    # start past its last row
        assert ld(FAKE, FAKE, 0, 128, 128, 128, 128, STREAM) == 1
        assert ld(FAKE, FAKE, 0, 0, 0, 128, 128, STREAM) == 1        # empty matrix
        assert ld(FAKE, FAKE, 0, 0, 128, 128, 0, STREAM) == 1        # stride
        st = p.store_tile(32, 128, half)
        assert st(NUL, FAKE, 0, 0, 16, 16, 16, STREAM) == 3
        assert st(FAKE, FAKE, 0, -3, 16, 16, 16, STREAM) == 1
    rt = p.roundtrip()
    assert rt(FAKE, NUL, 0, 0, 8, 8, 8, STREAM) == 3
    assert rt(FAKE, FAKE, 0, 0, 8, -8, 8, STREAM) == 1
    init, upd, fin, fwd = (p.softmax_init(), p.softmax_update(), p.softmax_finalize(),
                           p.softmax_forward())
    assert init(NUL, FAKE, 4, STREAM) == 3
    assert init(FAKE, FAKE, 0, STREAM) == 1
    assert upd(FAKE, FAKE, FAKE, NUL, 4, STREAM) == 3
    assert upd(FAKE, FAKE, FAKE, FAKE, -1, STREAM) == 1
    assert fin(FAKE, FAKE, FAKE, NUL, 4, STREAM) == 3               # normalizer required
    assert fwd(NUL, FAKE, FAKE, 4, 4, 2, STREAM) == 3
    assert fwd(FAKE, FAKE, FAKE, 0, 4, 2, STREAM) == 1
    assert fwd(FAKE, FAKE, FAKE, 4, 0, 2, STREAM) == 1
    assert fwd(FAKE, FAKE, FAKE, 4, 4, 0, STREAM) == 1
