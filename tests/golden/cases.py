"""Golden cases: the reference's own test inputs (seed, distribution, shape,
flags) plus a few ragged shapes, shared by ``make_golden.py`` (which runs the
reference's CUDA library on them) and the CPU/GPU tests (which check the
oracle and the new library against the stored outputs).

Each entry cites the reference test it restates.  Inputs are regenerated
from the seed with the oracle's mt19937 generator; fp16/bf16 inputs are the
fp32 draws rounded to nearest (``__float2half`` / ``__float2bfloat16``, as in
tests/unit/test_dtype.cu:46-50 and :554-557).
"""

CASES = [
    # name, kind, dtype, B, H, N, D, seed, lo, hi, causal, tol, source
    ("fwd_basic_small", "fwd", "f32", 1, 1, 8, 32, 42, -1.0, 1.0, False, 1e-3,
     "tests/unit/test_forward.cu:121-176"),
    ("fwd_causal_hd128", "fwd", "f32", 2, 2, 16, 128, 123, -0.5, 0.5, True, 2e-3,
     "tests/unit/test_forward.cu:178-227"),
    ("fwd_lse", "fwd", "f32", 2, 2, 16, 64, 7, -1.0, 1.0, False, 1e-3,
     "tests/unit/test_forward.cu:233-281"),
    ("fwd_lse_causal", "fwd", "f32", 1, 2, 16, 32, 9, -1.0, 1.0, True, 1e-3,
     "tests/unit/test_forward.cu:285-333"),
    ("bwd_basic_small", "bwd", "f32", 1, 1, 8, 32, 42, -1.0, 1.0, False, 1e-3,
     "tests/unit/test_backward.cu:138-215"),
    ("bwd_causal_hd128", "bwd", "f32", 1, 2, 16, 128, 7, -0.25, 0.25, True, 2e-3,
     "tests/unit/test_backward.cu:217-286"),
    ("fwd_fp16_vs_fp32", "fwd", "f16", 1, 1, 16, 32, 42, -1.0, 1.0, False, 1e-2,
     "tests/unit/test_dtype.cu:24-102"),
    ("fwd_bf16_vs_fp32", "fwd", "bf16", 1, 1, 16, 32, 42, -1.0, 1.0, False, 2e-2,
     "tests/unit/test_dtype.cu:446-524"),
    ("bwd_fp16_vs_fp32", "bwd", "f16", 1, 1, 8, 32, 42, -1.0, 1.0, False, 1e-2,
     "tests/unit/test_dtype.cu:308-421"),
    ("bwd_bf16_vs_fp32", "bwd", "bf16", 1, 1, 8, 32, 42, -1.0, 1.0, False, 2e-2,
     "tests/unit/test_dtype.cu:614-732"),
    ("fwd_hd128_half_range", "fwd", "f32", 1, 1, 16, 128, 42, -0.5, 0.5, False, 1e-3,
     "tests/unit/test_dtype.cu:197-246"),
    ("fwd_causal_future", "fwd", "f32", 1, 1, 16, 32, 42, -1.0, 1.0, True, 1e-3,
     "tests/unit/test_causal_mask.cu:22-96"),
    ("fwd_multihead_large", "fwd", "f32", 1, 32, 512, 64, 101, -0.5, 0.5, True, 1e-3,
     "tests/unit/test_stress_edge_cases.cu:320-357"),
    # ragged shapes (not multiples of any tile size)
    ("fwd_ragged_f32", "fwd", "f32", 1, 2, 100, 64, 1, -1.0, 1.0, True, 1e-3, "ragged"),
    ("bwd_ragged_f32", "bwd", "f32", 1, 1, 37, 64, 2, -1.0, 1.0, True, 1e-3, "ragged"),
    ("fwd_ragged_bf16", "fwd", "bf16", 2, 2, 300, 128, 3, -1.0, 1.0, True, 2e-2, "ragged"),
    ("bwd_ragged_bf16", "bwd", "bf16", 1, 2, 130, 64, 4, -1.0, 1.0, True, 2e-2, "ragged"),
    ("fwd_ragged_f16", "fwd", "f16", 1, 3, 257, 32, 5, -1.0, 1.0, False, 1e-2, "ragged"),
]

FIELDS = ("name", "kind", "dtype", "B", "H", "N", "D", "seed", "lo", "hi", "causal", "tol",
          "source")


def as_dicts():
    return [dict(zip(FIELDS, c)) for c in CASES]


def inputs(case):
    """fp32 inputs (already rounded to the case's dtype) for a case dict."""
    import oracle

    shape = (case["B"], case["H"], case["N"], case["D"])
    count = 4 if case["kind"] == "bwd" else 3
    arrs = oracle.interleaved_uniform(shape, case["seed"], case["lo"], case["hi"], count)
    if case["dtype"] == "bf16":
        arrs = [oracle.round_bf16(a) for a in arrs]
    elif case["dtype"] == "f16":
        arrs = [oracle.round_f16(a) for a in arrs]
    return arrs
