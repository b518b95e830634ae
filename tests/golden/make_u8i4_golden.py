"""Known answers for the uint8 x int4 operand pair, from the reference's own
tools/int4_prefill_model.py Int4MmulReference (4x8 uint8 x 8x16 int4, packed two per byte):
``IXB_REFERENCE=<checkout> python tests/golden/make_u8i4_golden.py`` writes ``u8i4_kat.npz``."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("IXB_REFERENCE", ""))


def require_reference() -> None:
    """The generators read the reference's own sources: IXB_REFERENCE must name its checkout."""
    if not os.environ.get("IXB_REFERENCE") or not (REF / "src" / "ignite_xdna").is_dir():
        raise SystemExit("set IXB_REFERENCE to the reference checkout's root (the tree holding src/ignite_xdna)")


def main():
    require_reference()
    sys.path.insert(0, str(REF))     # tools/int4_prefill_model.py imports tools.xdna1_roofline
    try:
        import tools.int4_prefill_model as int4
    finally:
        sys.path.remove(str(REF))
    rng = np.random.default_rng(2468)
    out = {}
    for i in range(6):
        a = rng.integers(0, 256, size=(4, 8), dtype=np.uint8)
        if i == 0:
            a[:] = 255
        b = rng.integers(-8, 8, size=(8, 16), dtype=np.int8)
        if i == 0:
            b[:] = -8
        bp = int4.Int4WeightPacker.pack(b)
        out[f"a{i}"], out[f"b{i}_packed"] = a, bp
        out[f"c{i}"] = int4.Int4MmulReference.execute(a, bp).astype(np.int64)
    np.savez_compressed(HERE / "u8i4_kat.npz", **out)
    print("wrote", HERE / "u8i4_kat.npz")


if __name__ == "__main__":
    main()
