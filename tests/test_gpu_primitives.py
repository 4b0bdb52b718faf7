"""The primitive API (cuflash::kernels::*) on the GPU, the parity half of the
reference's tests/unit/test_{matmul,online_softmax,tile_io}.cu: every
exported instantiation against numpy (fp64) at the reference tests'
tolerances, and against the reference library built from its own sources
(oracle/_ref, when present): bit-identical for the matrix products and the
tile copies, within a few ulp for the softmax (exp/log of the same values,
different reduction order)."""

import ctypes

import numpy as np
import pytest

import cuflash_attn as cf
import oracle
from primitive_abi import MM_FORMS, MM_SHAPES, TILE_SHAPES, Primitives

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prims():
    ours = Primitives(cf.library_path())
    ref = Primitives(oracle.REF_LIB_PATH) if oracle.REF_LIB_PATH.exists() else None
    return ours, ref


def _dev(a, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda", dtype) if dtype is not None else t.to("cuda")


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _mm_expected(form, A, B, C0, scale):
    A, B = A.astype(np.float64), B.astype(np.float64)
    if form == "matmul_ABt":
        return scale * A @ B.T
    if form == "matmul_AtB":
        return scale * A.T @ B
    prod = scale * A @ B
    return C0.astype(np.float64) + prod if form == "matmul_AB_acc" else prod


@pytest.mark.parametrize("shape", MM_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("form", MM_FORMS)
def test_matmul(cuda, prims, form, shape):
    import torch

    M, N, K = shape
    rng = np.random.default_rng(M * 1000 + N * 10 + K)
    a_shape = (K, M) if form == "matmul_AtB" else (M, K)
    b_shape = (N, K) if form == "matmul_ABt" else (K, N)
    A = rng.uniform(-1, 1, a_shape).astype(np.float32)
    B = rng.uniform(-1, 1, b_shape).astype(np.float32)
    C0 = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(K))
    ours, ref = prims
    outs = []
    for lib in (ours, ref):
        if lib is None:
            continue
        dA, dB, dC = _dev(A), _dev(B), _dev(C0)
        assert lib.matmul(form, M, N, K)(_p(dA), _p(dB), _p(dC), float(scale), _stream()) == 0
        torch.cuda.synchronize()
        outs.append(dC.cpu().numpy())
    want = _mm_expected(form, A, B, C0, float(scale))
    np.testing.assert_allclose(outs[0], want, atol=1e-4 if K <= 64 else 1e-3)
    if len(outs) == 2:  # same fused multiply-add chain as the reference
        assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("tile", TILE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_load_and_store_tile(cuda, prims, tile, half):
    import torch

    R, C = tile
    rows, cols, stride = 100, 150, 160  # partial windows at the bottom / right edges
    rng = np.random.default_rng(R + C)
    src = rng.uniform(-4, 4, (rows, stride)).astype(np.float32)
    if half:
        src = src.astype(np.float16)
    ours, ref = prims
    for r0, c0 in ((0, 0), (rows - R // 2, 7), (13, cols - 5)):
        win = np.zeros((R, C), np.float32)
        sub = src[r0:min(r0 + R, rows), c0:min(c0 + C, cols)].astype(np.float32)
        win[:sub.shape[0], :sub.shape[1]] = sub
        # load: in-matrix elements widened exactly, the rest 0
        for lib in (ours, ref):
            if lib is None:
                continue
            d_src = _dev(src)
            d_dst = torch.full((R * C,), 7.0, device="cuda")
            rc = lib.load_tile(R, C, half)(_p(d_src), _p(d_dst), r0, c0, rows, cols, stride,
                                           _stream())
            assert rc == 0
            torch.cuda.synchronize()
            assert np.array_equal(d_dst.cpu().numpy().reshape(R, C), win)
        # store: only the in-matrix part of the window changes
        tile_vals = rng.uniform(-4, 4, (R, C)).astype(np.float32)
        results = []
        for lib in (ours, ref):
            if lib is None:
                continue
            dst0 = np.full((rows, stride), -1.0, np.float16 if half else np.float32)
            d_dst = _dev(dst0)
            d_tile = _dev(tile_vals)
            rc = lib.store_tile(R, C, half)(_p(d_tile), _p(d_dst), r0, c0, rows, cols, stride,
                                            _stream())
            assert rc == 0
            torch.cuda.synchronize()
            results.append(d_dst.cpu().numpy())
        want = np.full((rows, stride), -1.0, np.float16 if half else np.float32)
        h, w = min(R, rows - r0), min(C, cols - c0)
        want[r0:r0 + h, c0:c0 + w] = tile_vals[:h, :w].astype(want.dtype)
        assert np.array_equal(results[0], want)
        if len(results) == 2:
            assert np.array_equal(results[0], results[1])


def test_roundtrip_copies_the_window(cuda, prims):
    import torch

    rows, cols, stride = 90, 70, 72
    src = np.random.default_rng(3).standard_normal((rows, stride)).astype(np.float32)
    ours, _ = prims
    d_src = _dev(src)
    d_dst = torch.zeros((rows, stride), device="cuda")
    assert ours.roundtrip()(_p(d_src), _p(d_dst), 40, 20, rows, cols, stride, _stream()) == 0
    torch.cuda.synchronize()
    want = np.zeros_like(src)
    want[40:90, 20:70] = src[40:90, 20:70]
    assert np.array_equal(d_dst.cpu().numpy(), want)


def test_online_softmax_state_primitives(cuda, prims):
    """init, two updates and finalize against the algebra in fp64, and the
    reference library's own primitives."""
    import torch

    rows = 1000
    rng = np.random.default_rng(11)
    bm1, bm2 = rng.uniform(-5, 5, rows).astype(np.float32), rng.uniform(-5, 5, rows).astype(np.float32)
    bs1, bs2 = rng.uniform(0.5, 40, rows).astype(np.float32), rng.uniform(0.5, 40, rows).astype(np.float32)
    m = np.maximum(bm1.astype(np.float64), bm2)
    l = bs1 * np.exp(bm1 - m) + bs2 * np.exp(bm2 - m)
    want_lse, want_norm = m + np.log(l), 1.0 / l
    got = []
    for lib in prims:
        if lib is None:
            continue
        sm, sl = (torch.empty(rows, device="cuda") for _ in range(2))
        lse, norm = (torch.empty(rows, device="cuda") for _ in range(2))
        s = _stream()
        assert lib.softmax_init()(_p(sm), _p(sl), rows, s) == 0
        assert lib.softmax_update()(_p(_dev(bm1)), _p(_dev(bs1)), _p(sm), _p(sl), rows, s) == 0
        assert lib.softmax_update()(_p(_dev(bm2)), _p(_dev(bs2)), _p(sm), _p(sl), rows, s) == 0
        assert lib.softmax_finalize()(_p(sm), _p(sl), _p(lse), _p(norm), rows, s) == 0
        torch.cuda.synchronize()
        got.append((lse.cpu().numpy(), norm.cpu().numpy()))
    np.testing.assert_allclose(got[0][0], want_lse, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(got[0][1], want_norm, rtol=1e-6)
    if len(got) == 2:
        np.testing.assert_allclose(got[0][0], got[1][0], rtol=4e-7, atol=1e-6)
        np.testing.assert_allclose(got[0][1], got[1][1], rtol=4e-7)


@pytest.mark.parametrize("rows,cols,block,lo,hi", [
    (64, 128, 32, -5.0, 5.0),     # reference Forward_LargeInput
    (3, 96, 64, -8.0, 8.0),       # reference Forward_MultiBlockCrossWarp
    (2, 4, 2, -1.0, 1.0),         # reference Forward_Basic (tiny)
    (5, 1000, 128, -30.0, 30.0),  # long rows, wide range
    (300, 33, 16, 80.0, 90.0),    # large values: stability
    (1, 1, 1, -3.0, -3.0),        # a single element
])
def test_online_softmax_forward(cuda, prims, rows, cols, block, lo, hi):
    import torch

    x = np.random.default_rng(rows * cols).uniform(lo, hi, (rows, cols)).astype(np.float32)
    x64 = x.astype(np.float64)
    mx = x64.max(1, keepdims=True)
    e = np.exp(x64 - mx)
    want = e / e.sum(1, keepdims=True)
    want_lse = (mx + np.log(e.sum(1, keepdims=True)))[:, 0]
    got = []
    for lib in prims:
        if lib is None:
            continue
        d_in = _dev(x)
        d_out = torch.empty_like(d_in)
        d_lse = torch.empty(rows, device="cuda")
        assert lib.softmax_forward()(_p(d_in), _p(d_out), _p(d_lse), rows, cols, block,
                                     _stream()) == 0
        torch.cuda.synchronize()
        got.append((d_out.cpu().numpy(), d_lse.cpu().numpy()))
    out, lse = got[0]
    np.testing.assert_allclose(out, want, atol=1e-4)      # the reference tests' bar
    np.testing.assert_allclose(out.sum(1), 1.0, atol=1e-5)
    np.testing.assert_allclose(lse, want_lse, rtol=1e-6, atol=1e-5)
    if len(got) == 2:
        np.testing.assert_allclose(out, got[1][0], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(lse, got[1][1], rtol=1e-6, atol=1e-5)
