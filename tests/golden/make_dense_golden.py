"""Golden fixture for the dense detect decode, from the reference's own decode_yolo_predictions.

Run with ``IXB_REFERENCE`` set to the reference checkout's root:
``IXB_REFERENCE=<checkout> python tests/golden/make_dense_golden.py`` writes ``dense_golden.npz``.

The heads are the seeded YOLOv8n graph's own int8 heads at 96x96 for two images (the CPU oracle
computes them; levels of 12x12, 6x6 and 3x3 anchors). The reference's
``runtime/session.py`` ``InferenceSession.decode_yolo_predictions`` (:1223-1278) is loaded by
file path with stand-ins for the NPU-only modules it imports at the top (``driver``, ``parity``,
``ring_scheduler``; its ``heads`` module is the reference's own) and run on those heads; its
float32 [2, 84, 189] output is stored beside them.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("IXB_REFERENCE", ""))
sys.path[:0] = [str(REPO), str(REPO / "oracle")]

import ixb_oracle as O  # noqa: E402
from ignite_xdna_b200 import build_yolov8, random_images  # noqa: E402
from ignite_xdna_b200.heads import HEAD_NAMES  # noqa: E402

IMGSZ = 96


def require_reference() -> None:
    """The generator reads the reference's own sources: IXB_REFERENCE must name its checkout."""
    if not os.environ.get("IXB_REFERENCE") or not (REF / "src" / "ignite_xdna").is_dir():
        raise SystemExit("set IXB_REFERENCE to the reference checkout's root (the tree holding src/ignite_xdna)")


def load_reference_session():
    for name in ("ignite_xdna", "ignite_xdna.runtime"):
        mod = types.ModuleType(name)
        mod.__path__ = []
        sys.modules.setdefault(name, mod)
    stubs = {"driver": ("XrtSiliconHarness", "setup_xrt_environment", "get_repo_root"),
             "parity": ("unblock_aie2_egress",),
             "ring_scheduler": ("BufferSet", "profile_pipelined_hardware_execution")}
    for mod_name, names in stubs.items():
        m = types.ModuleType(f"ignite_xdna.runtime.{mod_name}")
        for n in names:
            setattr(m, n, None)
        sys.modules[m.__name__] = m
    for name in ("heads", "session"):
        spec = importlib.util.spec_from_file_location(f"ignite_xdna.runtime.{name}",
                                                      REF / "src/ignite_xdna/runtime" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
    return sys.modules["ignite_xdna.runtime.session"]


def main():
    require_reference()
    S = load_reference_session()
    ir = build_yolov8("n", imgsz=IMGSZ)
    imgs = random_images(2, IMGSZ, seed=61)
    tensors = [O.run_image(ir, im) for im in imgs]
    heads = {n: np.concatenate([O.heads_int8(ir, t)[n] for t in tensors]) for n in HEAD_NAMES}
    tensor_of = dict(ir.outputs)
    scales = {n: (float(ir.tensors[tensor_of[n]].scale), 0) for n in HEAD_NAMES}
    out = S.InferenceSession.decode_yolo_predictions(dict(heads, scales=scales))
    egress = np.concatenate([heads[n].reshape(2, -1) for n in HEAD_NAMES], axis=1)
    offsets = np.cumsum([0] + [heads[n][0].size for n in HEAD_NAMES])[:-1]
    np.savez_compressed(HERE / "dense_golden.npz", egress=egress.astype(np.int8), out=out.astype(np.float32),
                        names=np.array(HEAD_NAMES), offsets=offsets.astype(np.int64),
                        scales=np.array([scales[n][0] for n in HEAD_NAMES], dtype=np.float64),
                        shapes=np.array([heads[n].shape[1:] for n in HEAD_NAMES], dtype=np.int64),
                        imgsz=np.int64(IMGSZ))
    print("wrote", HERE / "dense_golden.npz", out.shape)


if __name__ == "__main__":
    main()
