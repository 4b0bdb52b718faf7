"""The reference's own consumers of the C ABI, run unmodified against this
repository's library (the drop-in claim, tested the way a user of the
reference would find it).

* tests/integration/test_api_smoke.cpp of the reference: its host-only C++
  smoke test, compiled against this repository's include/ and linked with
  libcuflash_attn.so (the C++ overloads with their default stream argument,
  the enum, get_error_string and the C entry points); runs without a GPU.
* tests/integration/test_pytorch_comparison.py of the reference: its nine
  ctypes tests against PyTorch's scaled_dot_product_attention (fp32, fp16,
  bf16; forward, backward, causal), pointed at this library through the
  reference's own CUFLASH_LIB override; needs a GPU.

Both files are copied verbatim from the reference tree into oracle/_ref/
consumers/ by `make -C oracle consumers` (part of __graft_entry__.build());
the tests skip where that copy is absent.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

import cuflash_attn as cf

ROOT = Path(__file__).resolve().parents[1]
CONSUMERS = ROOT / "oracle" / "_ref" / "consumers"
CUDA_INC = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"


def _consumer(name):
    p = CONSUMERS / name
    if not p.exists():
        pytest.skip(f"{p} absent (make -C oracle consumers copies it from the reference tree)")
    return p


def test_reference_api_smoke_against_this_library(tmp_path):
    src = _consumer("test_api_smoke.cpp")
    lib_dir = Path(cf.library_path()).parent
    exe = tmp_path / "api_smoke"
    subprocess.run(["g++", "-std=c++17", "-O1", str(src), f"-I{ROOT / 'include'}",
                    f"-I{CUDA_INC}", f"-L{lib_dir}", "-lcuflash_attn",
                    f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "API smoke test passed" in r.stdout


@pytest.mark.gpu
def test_reference_pytorch_comparison_against_this_library(cuda):
    script = _consumer("test_pytorch_comparison.py")
    env = dict(os.environ, CUFLASH_LIB=str(Path(cf.library_path()).resolve()))
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True,
                       timeout=900, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "Results: 9 passed, 0 failed" in out, out[-4000:]
