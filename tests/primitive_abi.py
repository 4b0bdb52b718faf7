"""ctypes access to the cuflash::kernels primitive API (C++ symbols) of a
library, by demangled signature.  On x86-64 these functions take pointers,
ints and floats and return an int-sized enum, so ctypes calls them as it
would C functions."""

import ctypes
import subprocess

_P, _I, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float

MM_FORMS = ("matmul_ABt", "matmul_AB", "matmul_AB_acc", "matmul_AtB")
MM_SHAPES = [(64, 64, 32), (32, 32, 32), (64, 64, 64), (32, 32, 128), (64, 64, 128),
             (32, 64, 32), (32, 64, 64), (64, 32, 64)]
TILE_SHAPES = [(64, 64), (32, 32), (64, 32), (32, 64), (64, 128), (32, 128)]


def _table(path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True,
                         text=True, check=True).stdout
    mangled = [ln.split()[-1] for ln in out.splitlines() if "kernels" in ln]
    dem = subprocess.run(["c++filt"], input="\n".join(mangled), capture_output=True, text=True,
                         check=True).stdout.splitlines()
    table = {}
    for m, d in zip(mangled, dem):
        d = d.replace("cuflash::FlashAttentionError ", "", 1)
        table[d] = m
    return table


class Primitives:
    def __init__(self, path):
        self.cdll = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        self.table = _table(path)

    def _fn(self, demangled, argtypes):
        f = getattr(self.cdll, self.table[demangled])
        f.argtypes = argtypes
        f.restype = _I
        return f

    def matmul(self, form, M, N, K):
        name = (f"cuflash::kernels::{form}<{M}, {N}, {K}>(float const*, float const*, float*, "
                "float, CUstream_st*)")
        return self._fn(name, [_P, _P, _P, _F, _P])

    def load_tile(self, R, C, half=False):
        src = "__half const*" if half else "float const*"
        return self._fn(f"cuflash::kernels::load_tile<{R}, {C}>({src}, float*, int, int, int, "
                        "int, int, CUstream_st*)", [_P, _P] + [_I] * 5 + [_P])

    def store_tile(self, R, C, half=False):
        dst = "__half*" if half else "float*"
        return self._fn(f"cuflash::kernels::store_tile<{R}, {C}>(float const*, {dst}, int, int, "
                        "int, int, int, CUstream_st*)", [_P, _P] + [_I] * 5 + [_P])

    def roundtrip(self, R=64, C=64):
        return self._fn(f"cuflash::kernels::load_store_tile_roundtrip<{R}, {C}>(float const*, "
                        "float*, int, int, int, int, int, CUstream_st*)", [_P, _P] + [_I] * 5 + [_P])

    def softmax_init(self):
        return self._fn("cuflash::kernels::online_softmax_init(float*, float*, int, CUstream_st*)",
                        [_P, _P, _I, _P])

    def softmax_update(self):
        return self._fn("cuflash::kernels::online_softmax_update(float const*, float const*, "
                        "float*, float*, int, CUstream_st*)", [_P] * 4 + [_I, _P])

    def softmax_finalize(self):
        return self._fn("cuflash::kernels::online_softmax_finalize(float const*, float const*, "
                        "float*, float*, int, CUstream_st*)", [_P] * 4 + [_I, _P])

    def softmax_forward(self):
        return self._fn("cuflash::kernels::online_softmax_forward(float const*, float*, float*, "
                        "int, int, int, CUstream_st*)", [_P] * 3 + [_I] * 3 + [_P])
