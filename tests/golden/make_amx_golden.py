"""Generate tests/golden/golden_amx.npz: lowbit's own AMX repack (pack_amx,
src/lowbit/formats.py:275-293) of seeded int4 weights, so that the CPU tests
can check lowbit_b200.pack_amx and its inverse byte for byte without the
reference checkout. Run where the reference is importable:

    python tests/golden/make_amx_golden.py [path/to/lowbit/src]

(default: LOWBIT_REF_SRC, else a `reference` checkout beside this repository)."""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SHAPES = [(37, 300, True), (16, 128, False), (50, 1000, True), (3, 256, False)]


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from lowbit.formats import pack_amx, quantize_int4  # the reference package
    out = {}
    for i, (n, k, asym) in enumerate(SHAPES):
        w = np.random.default_rng(100 + i).standard_normal((n, k)).astype(np.float32)
        W = quantize_int4(w, asym=asym)
        A = pack_amx(W)
        out[f"a{i}_w"] = w
        for f in ("qw", "scales", "sz", "zeros"):
            out[f"a{i}_{f}"] = getattr(A, f)
    np.savez_compressed(HERE / "golden_amx.npz", **out)
    print("wrote", HERE / "golden_amx.npz")


if __name__ == "__main__":
    default = os.environ.get("LOWBIT_REF_SRC", str(HERE.parents[2] / "reference" / "src"))
    main(sys.argv[1] if len(sys.argv) > 1 else default)
