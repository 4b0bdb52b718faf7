import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for sub in ("cuflash-attn_b200", "oracle", "tests/golden", "tests"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def lib():
    import cuflash_attn

    return cuflash_attn.CuFlashAttn()


@pytest.fixture(scope="session")
def ref_lib():
    """The reference library built from its own sources (oracle/_ref)."""
    import cuflash_attn
    import oracle

    if not oracle.REF_LIB_PATH.exists():
        pytest.skip("reference build oracle/_ref/libcuflash_attn_ref.so is absent")
    return cuflash_attn.CuFlashAttn(str(oracle.REF_LIB_PATH), reference_abi_only=True)


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def parity_record():
    """Records the margins of the low-precision parity checks: each call
    appends one row (test, tensor, e = error vs fp64, e_ref = the reference
    library's error on the same inputs, allowance = how far e may exceed
    e_ref).  With CUFLASH_PARITY_RECORD=<path> the rows are written there as
    JSON lines when the session ends (summarised in profiles/parity_margin.md)."""
    rows = []

    def add(test, tensor, e, e_ref, allowance):
        rows.append({"test": test, "tensor": tensor, "e": float(e), "e_ref": float(e_ref),
                     "allowance": float(allowance),
                     "used": (float(e) - float(e_ref)) / float(allowance) if allowance else None})

    yield add
    path = os.environ.get("CUFLASH_PARITY_RECORD")
    if path and rows:
        with open(path, "a") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")
