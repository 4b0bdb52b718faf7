"""Forward parity on the GPU, through the C ABI.

Bars:
* fp32: within 1e-4 absolute of the fp64 ground truth on O and L;
* fp16/bf16: within 2e-2 absolute of fp64, and no worse than the reference
  library's own error on the same inputs (when oracle/_ref is present);
* the reference tests' golden outputs (tests/golden) within each test's
  tolerance.
"""

from pathlib import Path

import numpy as np
import pytest

import cases
import oracle
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_outputs.npz"
LOWP_TOL = 2e-2
F32_TOL = 1e-4
# How far the error may exceed the reference library's own on the same
# inputs.  Both libraries round P to the input dtype before PV and O once at
# the store; they differ in how P is rounded (ex2.approx and a running
# maximum raised in steps here, expf and the exact maximum there), which can
# flip one output rounding.  Measured (profiles/parity_margin.md): causal
# cases match the reference's error exactly; non-causal bf16 exceeds it by up
# to 4.8e-4 (half a bf16 ulp at |O| = 0.25 is 9.8e-4), fp16 by up to 2.3e-5,
# L by up to 3.5e-7.
REF_SLACK_O = {"bf16": 1e-3, "f16": 1e-4}
REF_SLACK_L = 1e-5


def run_fwd(lib, arrs, dt, causal, scale):
    Q, K, V = (to_dev(a, dt) for a in arrs[:3])
    O, L = lib.forward(Q, K, V, causal=causal, scale=scale)
    import torch

    torch.cuda.synchronize()
    if hasattr(lib.lib, "cuflash_device_status"):
        assert lib.device_status() == 0
    return host(O), host(L)


@pytest.mark.parametrize("case", [c for c in cases.as_dicts() if c["kind"] == "fwd"],
                         ids=lambda c: c["name"])
def test_forward_golden(lib, cuda, case):
    arrs = cases.inputs(case)
    scale = 1.0 / np.sqrt(case["D"])
    O, L = run_fwd(lib, arrs, case["dtype"], case["causal"], scale)
    O64, L64 = oracle.forward_f64(*arrs[:3], scale, case["causal"])
    bar = F32_TOL if case["dtype"] == "f32" else LOWP_TOL
    assert max_err(O, O64) < bar
    assert max_err(L, L64) < bar
    if GOLDEN.exists():
        g = np.load(GOLDEN)
        gO, gL = g[case["name"] + "/O"], g[case["name"] + "/L"]
        assert max_err(O[:, :gO.shape[1]], gO) < case["tol"]
        assert max_err(L[:, :gL.shape[1]], gL) < case["tol"]


SHAPES = [
    # B, H, N, D
    (1, 1, 1, 32), (1, 1, 7, 64), (1, 2, 128, 128), (2, 1, 129, 64), (1, 1, 255, 32),
    (1, 2, 256, 128), (2, 2, 300, 128), (1, 1, 513, 64), (1, 2, 1024, 128), (1, 1, 1000, 32),
]


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_forward_lowp_vs_f64_and_reference(lib, ref_lib, cuda, parity_record, request, dt,
                                           causal, shape):
    B, H, N, D = shape
    seed = 1000 + N * 7 + D + (1 if causal else 0)
    Q, K, V = (round_to(oracle.normal(shape, seed + i), dt) for i in range(3))
    scale = 1.0 / np.sqrt(D)
    O, L = run_fwd(lib, (Q, K, V), dt, causal, scale)
    O64, L64 = oracle.forward_f64(Q, K, V, scale, causal)
    eO, eL = max_err(O, O64), max_err(L, L64)
    assert eO < LOWP_TOL and eL < LOWP_TOL, (eO, eL)
    Or, Lr = run_fwd(ref_lib, (Q, K, V), dt, causal, scale)
    rO, rL = max_err(Or, O64), max_err(Lr, L64)
    parity_record(request.node.name, "O", eO, rO, REF_SLACK_O[dt])
    parity_record(request.node.name, "L", eL, rL, REF_SLACK_L)
    assert eO <= rO + REF_SLACK_O[dt], (eO, rO)
    assert eL <= rL + REF_SLACK_L, (eL, rL)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(2, 8, 1024, 64), (1, 2, 100, 32), (1, 1, 333, 128)],
                         ids=lambda s: "x".join(map(str, s)))
def test_forward_f32_within_1e4(lib, cuda, causal, shape):
    # BASELINE config 1 is (2, 8, 1024, 64) causal, U[-1,1], seeds 1/2/3
    Q, K, V = (oracle.uniform(shape, s) for s in (1, 2, 3))
    scale = 1.0 / np.sqrt(shape[3])
    O, L = run_fwd(lib, (Q, K, V), "f32", causal, scale)
    O64, L64 = oracle.forward_f64(Q, K, V, scale, causal)
    assert max_err(O, O64) < F32_TOL
    assert max_err(L, L64) < F32_TOL


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_forward_f32_shapes(lib, cuda, causal, shape):
    """3xTF32 forward at every head_dim and ragged length, N(0,1) inputs:
    long enough at head_dim 128 (up to 32 K/V blocks) that every ring stage,
    the one in Q's shared-memory region included, is refilled many times."""
    D = shape[3]
    Q, K, V = (oracle.normal(shape, 700 + shape[2] + D + i) for i in range(3))
    scale = 1.0 / np.sqrt(D)
    O, L = run_fwd(lib, (Q, K, V), "f32", causal, scale)
    O64, L64 = oracle.forward_f64(Q, K, V, scale, causal)
    assert max_err(O, O64) < F32_TOL, max_err(O, O64)
    assert max_err(L, L64) < F32_TOL, max_err(L, L64)


def test_config2_forward_sampled_units(lib, cuda):
    """BASELINE config 2 (fp16, B4 H16 N2048 D128, non-causal): the whole
    problem runs on the GPU, a sample of (b,h) units is checked in fp64."""
    import torch

    shape = (4, 16, 2048, 128)
    arrs = [round_to(oracle.normal(shape, s), "f16") for s in (11, 12, 13)]
    scale = 1.0 / np.sqrt(128)
    O, L = run_fwd(lib, arrs, "f16", False, scale)
    for u in (0, 37, 63):
        b, h = divmod(u, 16)
        sub = [a[b:b + 1, h:h + 1] for a in arrs]
        O64, L64 = oracle.forward_f64(*sub, scale, False)
        assert max_err(O[b, h], O64[0, 0]) < LOWP_TOL
        assert max_err(L[b, h], L64[0, 0]) < LOWP_TOL
    del torch


def test_config3_forward_sampled_units(lib, cuda):
    """BASELINE config 3 (bf16 causal, B8 H32 N4096 D128, inputs 0.5*N(0,1))."""
    shape = (8, 32, 4096, 128)
    arrs = [round_to(oracle.normal(shape, s, std=0.5), "bf16") for s in (21, 22, 23)]
    scale = 1.0 / np.sqrt(128)
    O, L = run_fwd(lib, arrs, "bf16", True, scale)
    for u in (0, 255):
        b, h = divmod(u, 32)
        sub = [a[b:b + 1, h:h + 1] for a in arrs]
        O64, L64 = oracle.forward_f64(*sub, scale, True)
        assert max_err(O[b, h], O64[0, 0]) < LOWP_TOL
        assert max_err(L[b, h], L64[0, 0]) < LOWP_TOL
    assert np.all(np.isfinite(O)) and np.all(np.isfinite(L))


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_causal_future_independence(lib, cuda, dt):
    # tests/unit/test_causal_mask.cu:22-96, at a multi-tile length
    shape = (1, 2, 640, 64)
    Q, K, V = (round_to(oracle.uniform(shape, s), dt) for s in (1, 2, 3))
    O1, _ = run_fwd(lib, (Q, K, V), dt, True, 0.125)
    K2, V2 = K.copy(), V.copy()
    K2[:, :, 320:] = round_to(K2[:, :, 320:] + 0.5, dt)
    V2[:, :, 320:] = round_to(V2[:, :, 320:] - 0.5, dt)
    O2, _ = run_fwd(lib, (Q, K2, V2), dt, True, 0.125)
    assert max_err(O1[:, :, :320], O2[:, :, :320]) < 1e-5


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_numerical_stability(lib, cuda, dt):
    # tests/unit/test_numerical_stability.cu: constant 100, tiny values, +-50 mix
    shape = (1, 1, 16, 32)
    big = np.full(shape, 100.0, np.float32)
    O, L = run_fwd(lib, (big, big, big), dt, False, 1 / np.sqrt(32))
    assert np.all(np.isfinite(O)) and np.all(np.isfinite(L))
    assert max_err(O, 100.0) < 1e-3
    tiny = np.full(shape, 1e-4, np.float32)
    O, L = run_fwd(lib, (tiny, tiny, tiny), dt, False, 1 / np.sqrt(32))
    assert np.all(np.isfinite(O)) and np.all(np.isfinite(L))
    mix = np.where(np.arange(np.prod(shape)).reshape(shape) % 3 == 0, 50.0,
                   np.where(np.arange(np.prod(shape)).reshape(shape) % 3 == 1, -50.0, 0.001))
    mix = mix.astype(np.float32)
    O, L = run_fwd(lib, (mix, mix, mix), dt, False, 1 / np.sqrt(32))
    assert np.all(np.isfinite(O)) and np.all(np.isfinite(L))


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_causal_seq_len_one_equals_noncausal(lib, cuda, dt):
    # tests/unit/test_stress_edge_cases.cu:359-400
    shape = (2, 3, 1, 128)
    Q, K, V = (round_to(oracle.uniform(shape, s), dt) for s in (7, 8, 9))
    a = run_fwd(lib, (Q, K, V), dt, True, 0.1)
    b = run_fwd(lib, (Q, K, V), dt, False, 0.1)
    assert max_err(a[0], b[0]) < 1e-5 and max_err(a[1], b[1]) < 1e-5


def test_scale_zero_is_uniform_average(lib, cuda):
    shape = (1, 1, 300, 64)
    Q, K, V = (round_to(oracle.uniform(shape, s), "bf16") for s in (4, 5, 6))
    O, L = run_fwd(lib, (Q, K, V), "bf16", True, 0.0)
    csum = np.cumsum(V[0, 0].astype(np.float64), axis=0) / np.arange(1, 301)[:, None]
    assert max_err(O[0, 0], csum) < 1e-2
    assert max_err(L[0, 0], np.log(np.arange(1, 301))) < 1e-4


def test_repeated_calls_do_not_leak(lib, cuda):
    # tests/unit/test_stress_edge_cases.cu:264-309
    import torch

    shape = (1, 4, 512, 128)
    Q, K, V = (to_dev(oracle.uniform(shape, s), "bf16") for s in (1, 2, 3))
    lib.forward(Q, K, V, causal=True)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    O = torch.empty_like(Q)
    L = torch.empty(shape[:3], device="cuda", dtype=torch.float32)
    for _ in range(50):
        lib.forward(Q, K, V, causal=True, O=O, L=L)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert abs(free0 - free1) < (1 << 20)
