"""Shared helpers for the GPU parity tests."""

import numpy as np

TORCH_DT = None


def torch_dtype(name):
    import torch

    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


def round_to(a, name):
    import oracle

    if name == "bf16":
        return oracle.round_bf16(a)
    if name == "f16":
        return oracle.round_f16(a)
    return np.asarray(a, np.float32)


def to_dev(a, name):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda", torch_dtype(name))


def host(t):
    return t.float().cpu().numpy()


def max_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0
