"""Golden fixtures for the GPU decode, from the reference's own decode.

Run with ``IXB_REFERENCE`` set to the reference checkout's root:
``python tests/golden/make_decode_golden.py``. It
* loads the reference's ``pipelines/decode_native.py`` table builders by file path (its package
  and its native-library import stubbed out) and records sha256 of the tables they make for the
  engine's head scales, which pins ``ignite_xdna_b200.decode``'s restated builders;
* builds the reference's ``decode_native.c`` (oracle/build_ref.sh) and runs ``yolo_decode_int8``
  on the heads of a 160x160 YOLOv8n run (the oracle's), several letterboxes and thresholds;
* writes ``decode_golden.npz`` (heads, letterboxes, thresholds, detections) and
  ``decode_tables.json`` (table hashes).
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import subprocess
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("IXB_REFERENCE", ""))


def require_reference() -> None:
    """The generators read the reference's own sources: IXB_REFERENCE must name its checkout."""
    if not os.environ.get("IXB_REFERENCE") or not (REF / "src" / "ignite_xdna").is_dir():
        raise SystemExit("set IXB_REFERENCE to the reference checkout's root (the tree holding src/ignite_xdna)")
sys.path[:0] = [str(REPO), str(REPO / "oracle"), str(HERE)]

import ixb_oracle as O  # noqa: E402
import ref_decode  # noqa: E402
from ignite_xdna_b200 import build_yolov8, random_images  # noqa: E402
from ignite_xdna_b200 import decode as D  # noqa: E402
from ignite_xdna_b200.heads import HEAD_NAMES, DetectHeadLayout, HeadSpec  # noqa: E402
from ignite_xdna_b200.plan import build_plan  # noqa: E402

IMGSZ = 160
CASES = [(0.25, 0.5, (0.0, 0.0, 1.0)), (0.5, 0.45, (12.0, 0.0, 0.5)), (0.1, 0.7, (3.5, 7.25, 1.25))]


def load_ref_tables():
    for name in ("ignite_xdna", "ignite_xdna.pipelines"):
        mod = types.ModuleType(name)
        mod.__path__ = []
        sys.modules.setdefault(name, mod)
    pre = types.ModuleType("ignite_xdna.pipelines.preprocess")
    pre._compile_native_dll = lambda *a, **k: False      # the reference's own library stays unbuilt here
    sys.modules["ignite_xdna.pipelines.preprocess"] = pre
    spec = importlib.util.spec_from_file_location("ignite_xdna.pipelines.decode_native",
                                                  REF / "src/ignite_xdna/pipelines/decode_native.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest() if a is not None else "none"


def main():
    require_reference()
    subprocess.run(["sh", str(REPO / "oracle" / "build_ref.sh")], check=True)
    R = load_ref_tables()
    lib = ref_decode.load()
    ir = build_yolov8("n", imgsz=IMGSZ)
    dp = build_plan(ir, 4)
    tensor_of = dict(ir.outputs)
    layout = DetectHeadLayout(tuple(HeadSpec(n, (ir.tensors[tensor_of[n]].channels, ir.tensors[tensor_of[n]].height,
                                                 ir.tensors[tensor_of[n]].width), dp.head_offsets[n],
                                             ir.tensors[tensor_of[n]].scale, 0) for n in HEAD_NAMES),
                              dp.egress_image_bytes)
    imgs = random_images(4, IMGSZ, seed=77)
    heads = O.run_batch_egress(ir, imgs)
    anchors = D.anchor_grid(IMGSZ)
    hashes = {}
    for name in HEAD_NAMES:
        s = layout.spec(name)
        if name.endswith("box"):
            hashes[f"{name}_dfl"] = sha(R.dfl_exp_table(s.scale, 0))
        else:
            sig = R.sigmoid_table(s.scale, 0)
            hashes[f"{name}_sigmoid"] = sha(sig)
            hashes[f"{name}_low"] = sha(R.sigmoid_low_table(sig))
    out = {"heads": heads, "anchors_x": anchors[0], "anchors_y": anchors[1], "strides": anchors[2]}
    for ci, (conf, iou, lb) in enumerate(CASES):
        tables = []
        for bname, cname in D.HEAD_PAIRS:
            bs, cs = layout.spec(bname), layout.spec(cname)
            sig = R.sigmoid_table(cs.scale, 0)
            tables.append((R.dfl_exp_table(bs.scale, 0), sig, R.sigmoid_low_table(sig),
                           float(np.log(min(max(conf, 1e-12), 1 - 1e-12) / (1 - min(max(conf, 1e-12), 1 - 1e-12)))
                                 / float(cs.scale))))
        for i in range(heads.shape[0]):
            b, s, c = ref_decode.decode(lib, heads[i], layout, tables, anchors, conf, iou, lb)
            out[f"c{ci}_i{i}_boxes"], out[f"c{ci}_i{i}_scores"], out[f"c{ci}_i{i}_classes"] = b, s, c
            print(f"case {ci} image {i}: {len(s)} detections")
    out["cases"] = np.array([[c, u, *lb] for c, u, lb in CASES], dtype=np.float64)
    np.savez_compressed(HERE / "decode_golden.npz", **out)
    (HERE / "decode_tables.json").write_text(json.dumps({"imgsz": IMGSZ, "tables": hashes}, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
