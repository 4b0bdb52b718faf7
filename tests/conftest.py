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
