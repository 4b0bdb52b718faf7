"""Generates tests/golden/reference_outputs.npz by running the REFERENCE
library (AICL-Lab/cuflash-attn, compiled from its own sources into
oracle/_ref/libcuflash_attn_ref.so by ``make -C oracle ref``) on the golden
cases of cases.py.  Needs a GPU; run once and commit the .npz:

    python tests/golden/make_golden.py

For "fwd" cases it stores the reference's O and L; for "bwd" cases it runs
the reference's forward then backward and stores dQ, dK, dV (and O, L).
"""

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "cuflash-attn_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests" / "golden"))

import cases  # noqa: E402
import cuflash_attn  # noqa: E402
import oracle  # noqa: E402

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def main():
    ref = cuflash_attn.CuFlashAttn(str(oracle.REF_LIB_PATH), reference_abi_only=True)
    out = {}
    for c in cases.as_dicts():
        arrs = cases.inputs(c)
        dt = TORCH_DT[c["dtype"]]
        t = [torch.from_numpy(a).to("cuda", dt).contiguous() for a in arrs]
        scale = 1.0 / np.sqrt(c["D"])
        O, L = ref.forward(t[0], t[1], t[2], causal=c["causal"], scale=scale)
        torch.cuda.synchronize()
        out[c["name"] + "/O"] = O.float().cpu().numpy()
        out[c["name"] + "/L"] = L.cpu().numpy()
        if c["kind"] == "bwd":
            dQ, dK, dV = ref.backward(t[0], t[1], t[2], O, L, t[3], causal=c["causal"],
                                      scale=scale)
            torch.cuda.synchronize()
            out[c["name"] + "/dQ"] = dQ.float().cpu().numpy()
            out[c["name"] + "/dK"] = dK.float().cpu().numpy()
            out[c["name"] + "/dV"] = dV.float().cpu().numpy()
        print(c["name"], "ok", flush=True)
    # keep the fixture small: large outputs keep their first two heads only
    # (the tests compare the same slice)
    for k, v in list(out.items()):
        if v.size > (1 << 16):
            out[k] = np.ascontiguousarray(v[:, :2])
    dst = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).with_name(
        "reference_outputs.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst)


if __name__ == "__main__":
    main()
