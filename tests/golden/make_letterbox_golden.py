"""Golden hashes for the GPU letterbox, from the reference's own fused_preprocess_bgr_to_c8_plane.

``python tests/golden/make_letterbox_golden.py`` (reference tree present): builds the reference's
preprocessing (oracle/build_ref.sh), letterboxes seeded BGR frames of several sizes into 640x640
through the YOLOv8n input table, and writes ``letterbox_golden.json``: per case the sha256 of the
quantized plane (bytes 0..2 of each pixel, q domain) and the (pad_top, pad_left, scale) it returns.
"""
from __future__ import annotations

import hashlib
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path[:0] = [str(REPO), str(HERE)]

import ref_preprocess  # noqa: E402
from ignite_xdna_b200 import build_yolov8  # noqa: E402
from ignite_xdna_b200.plan import input_lut_t  # noqa: E402

CASES = [(640, 480, 1), (1280, 720, 2), (333, 517, 3), (640, 640, 4), (320, 200, 5), (1920, 1080, 6)]


def frame(w, h, seed):
    return np.random.default_rng(seed).integers(0, 256, size=(h, w, 3), dtype=np.uint8)


def main():
    subprocess.run(["sh", str(REPO / "oracle" / "build_ref.sh")], check=True)
    lib = ref_preprocess.load()
    ir = build_yolov8("n", imgsz=640)
    lut_q = (input_lut_t(ir.tensors[ir.input].scale).astype(np.int16) + 128).astype(np.uint8)
    out = []
    for w, h, seed in CASES:
        plane, (top, left, scale) = ref_preprocess.letterbox(lib, frame(w, h, seed), 640, 640, lut_q)
        out.append({"w": w, "h": h, "seed": seed, "sha256": hashlib.sha256(plane.tobytes()).hexdigest(),
                    "pad_top": top, "pad_left": left, "scale": float(np.float32(scale))})
        print(out[-1])
    (HERE / "letterbox_golden.json").write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
