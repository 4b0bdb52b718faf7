"""Failure detection without a GPU fault: a bounded wait that runs out.

The fp16/bf16 forward has two test options (cuflash_set_option): a wait
limit in milliseconds, and a switch that makes its first CTA leave out one
K load, so that the MMA thread's wait for that load can never complete.
The wait gives up after the limit, the kernel tears down (the producer
drains its issued loads, the TMEM is freed) and returns; the failure goes
to the family's device status word and to the host-mapped word every entry
point reads.  The next call of ANY entry point then returns CUDA_ERROR and
launches nothing, until cuflash_device_status() reads and clears the code;
after that the library computes correct results again.  The reference's
failure surface is launch errors and OOM only
(src/forward/flash_attention_forward_typed.cu:281-282); the bounded waits are
this library's, so this is where they are exercised.
"""

import ctypes
import time

import numpy as np
import pytest

import cuflash_attn as cf
import oracle
from helpers import host, max_err, round_to, to_dev

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 1  # kStatusWaitTimeout


def _raw_forward(lib, Q, K, V, O, L, causal=True):
    import torch

    B, H, N, D = Q.shape
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    return lib.lib.cuflash_attention_forward_bf16(
        p(Q), p(K), p(V), p(O), p(L), B, H, N, D, ctypes.c_float(D ** -0.5), causal,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_forward_wait_timeout_is_reported_then_cleared(lib, cuda):
    import torch

    B, H, N, D = 1, 2, 512, 128
    arrs = [round_to(oracle.normal((B, H, N, D), s), "bf16") for s in (81, 82, 83)]
    Q, K, V = (to_dev(x, "bf16") for x in arrs)
    # a normal call first (it also binds the host-visible status word)
    O_ref, L_ref = lib.forward(Q, K, V, causal=True)
    torch.cuda.synchronize()
    assert lib.device_status() == 0

    O = torch.zeros_like(Q)
    L = torch.zeros((B, H, N), device="cuda")
    lib.set_option("CUFLASH_TEST_WAIT_LIMIT_MS", 50)
    lib.set_option("CUFLASH_TEST_SKIP_K_LOAD", 1)
    try:
        t0 = time.monotonic()
        assert _raw_forward(lib, Q, K, V, O, L) == cf.SUCCESS  # the launch itself is fine
        torch.cuda.synchronize()  # the kernel returns: its waits are bounded
        elapsed = time.monotonic() - t0
    finally:
        lib.set_option("CUFLASH_TEST_WAIT_LIMIT_MS", -1)
        lib.set_option("CUFLASH_TEST_SKIP_K_LOAD", -1)
    assert elapsed < 5.0, elapsed
    try:
        # every entry point now refuses work, the forward and other families
        assert _raw_forward(lib, Q, K, V, O, L) == cf.CUDA_ERROR
        with pytest.raises(cf.CuFlashError) as e:
            lib.backward(Q, K, V, O_ref, L_ref, Q, causal=True)
        assert e.value.code == cf.CUDA_ERROR
        with pytest.raises(cf.CuFlashError):
            lib.decode(Q[:, :, :1].contiguous(), K, V)
    finally:
        code = lib.device_status()  # reads and clears
    assert code == WAIT_TIMEOUT
    assert lib.device_status() == 0
    # the library works again, with the same results as before
    O2, L2 = lib.forward(Q, K, V, causal=True)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    assert torch.equal(O2, O_ref) and torch.equal(L2, L_ref)
    O64, L64 = oracle.forward_f64(*arrs, D ** -0.5, True)
    assert max_err(host(O2), O64) < 2e-2 and max_err(host(L2), L64) < 2e-2


def test_other_ctas_of_the_failed_launch_finish_their_work(lib, cuda):
    """Only the CTA whose load was left out gives up: rows of the items the
    other CTAs own are computed as usual (and agree with a clean call)."""
    import torch

    B, H, N, D = 1, 4, 1024, 64
    arrs = [round_to(oracle.normal((B, H, N, D), s), "bf16") for s in (84, 85, 86)]
    Q, K, V = (to_dev(x, "bf16") for x in arrs)
    O_ref, L_ref = lib.forward(Q, K, V, causal=True)
    torch.cuda.synchronize()
    O = torch.full_like(Q, float("nan"))
    L = torch.full((B, H, N), float("nan"), device="cuda")
    lib.set_option("CUFLASH_TEST_WAIT_LIMIT_MS", 50)
    lib.set_option("CUFLASH_TEST_SKIP_K_LOAD", 1)
    try:
        assert _raw_forward(lib, Q, K, V, O, L) == cf.SUCCESS
        torch.cuda.synchronize()
    finally:
        lib.set_option("CUFLASH_TEST_WAIT_LIMIT_MS", -1)
        lib.set_option("CUFLASH_TEST_SKIP_K_LOAD", -1)
        code = lib.device_status()
    assert code == WAIT_TIMEOUT
    same = (O == O_ref).all(dim=-1)  # rows identical to the clean call
    assert not bool(torch.isnan(O).any())  # every row was written
    # all but the failed CTA's rows (at most one item of 256 rows) match
    assert int((~same).sum()) <= 256, int((~same).sum())
    assert float(same.float().mean()) > 0.5
    np.testing.assert_array_equal(host(L)[host(same.float()) > 0], host(L_ref)[host(same.float()) > 0])
