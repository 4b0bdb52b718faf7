"""Writes reference_symbols.txt: the dynamic symbols the reference library
exports (its C ABI, the C++ overloads and the cuflash::kernels primitive
API), read with `nm -D` from the reference built by `make -C oracle ref`.
The ABI tests require this library to export every one of them."""

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = HERE.parents[1] / "oracle" / "_ref" / "libcuflash_attn_ref.so"


def main() -> None:
    out = subprocess.run(["nm", "-D", "--defined-only", str(REF)], capture_output=True, text=True,
                         check=True).stdout
    names = sorted({ln.split()[-1] for ln in out.splitlines()
                    if len(ln.split()) == 3 and ln.split()[1] in ("T", "W")})
    (HERE / "reference_symbols.txt").write_text("\n".join(names) + "\n")
    print(len(names), "symbols")


if __name__ == "__main__":
    main()
