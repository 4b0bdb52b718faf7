"""The FMA-pipe 2^x used for one exponential pair in four by the backward
softmax (sm100.cuh: exp2_poly2): range reduction x = n + f with n = round(x)
and a degree-3 polynomial for 2^f on [-1/2, 1/2].  This restates the same
steps in float32 numpy with the coefficients read from the header and checks
the relative error against 2^x, so a changed coefficient or a broken
reduction fails here on CPU; the GPU backward tests check the kernels' end
results against fp64."""

import re
from pathlib import Path

import numpy as np

HDR = Path(__file__).resolve().parents[1] / "cuflash-attn_b200" / "csrc" / "sm100.cuh"


def _coeffs():
    src = HDR.read_text()
    body = src[src.index("exp2_poly2(float x0"):]
    body = body[:body.index("}\n")]
    vals = [float(v) for v in re.findall(r"f2_pack\((0\.\d+)f,", body)]
    # Horner order in the source: c3, c2, then c1, c0
    assert len(vals) == 4, vals
    return vals


def exp2_poly_f32(x):
    c3, c2, c1, c0 = (np.float32(v) for v in _coeffs())
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    f = (x - n).astype(np.float32)
    q = (f * c3 + c2).astype(np.float32)
    q = (q * f + c1).astype(np.float32)
    q = (q * f + c0).astype(np.float32)
    ti = t.view(np.int32)
    return (q.view(np.int32) + (ti << 23)).view(np.float32)


def test_exp2_poly_relative_error():
    x = np.linspace(-125.0, 1.0, 2_000_003, dtype=np.float64).astype(np.float32)
    y = exp2_poly_f32(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y - ref) / ref
    assert rel.max() < 1e-4, rel.max()


def test_exp2_poly_reduction_points():
    # integers and half-integers exercise the rounding of the reduction
    x = np.arange(-125.0, 1.01, 0.5, dtype=np.float32)
    y = exp2_poly_f32(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert (np.abs(y - ref) / ref).max() < 1e-4


def test_exp2_poly_clamps_masked_scores():
    # -inf (masked scores) clamps to 2^-125: below every bf16/fp16 P's resolution
    y = exp2_poly_f32(np.array([-np.inf, -1e30, -200.0], dtype=np.float32))
    assert np.all(y >= 0) and np.all(y < 1e-37)
