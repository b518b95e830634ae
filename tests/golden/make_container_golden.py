"""Golden fixtures for the .ignite container, from the reference's own serializer.

Run with ``IXB_REFERENCE`` set to the reference checkout's root:
``IXB_REFERENCE=<checkout> python tests/golden/make_container_golden.py``.

The reference's ``compiler/serializer.py`` (standard library only) is loaded by file path and
its ``IgniteModelWriter`` writes:

* the seeded YOLOv8n graph at 64x64 as this engine's container payload (the manifest and blobs
  of ``ignite_xdna_b200.container.graph_manifest``); only the file's SHA-256 and size are kept
  (``container_golden.json``), which the engine's own writer must reproduce byte for byte;
* a small container with an NPU-style manifest and three blobs (``container_ref_small.ignite``),
  which the engine's reader must parse.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("IXB_REFERENCE", ""))
sys.path[:0] = [str(REPO)]

from ignite_xdna_b200 import build_yolov8  # noqa: E402
from ignite_xdna_b200.container import ARCH_B200, graph_manifest  # noqa: E402

SMALL_MANIFEST = {"model_name": "small", "format_version": 1, "task": "detect", "input_shape": [1, 3, 64, 64],
                  "graph_engine": {"workspace_bytes": 4096, "layers": [{"index": 0, "name": "conv0"}]},
                  "strides": [8, 16, 32], "reg_max": 16}
SMALL_BLOBS = [("engine.xclbin", bytes(range(200)), "xclbin"), ("insts.bin", b"\x01\x02\x03" * 11,
                                                                   "npu_instructions"),
               ("wpackets.bin", bytes(64 * 3), "weight_packets")]


def require_reference() -> None:
    """The generator reads the reference's own sources: IXB_REFERENCE must name its checkout."""
    if not os.environ.get("IXB_REFERENCE") or not (REF / "src" / "ignite_xdna").is_dir():
        raise SystemExit("set IXB_REFERENCE to the reference checkout's root (the tree holding src/ignite_xdna)")


def load_serializer():
    spec = importlib.util.spec_from_file_location("ref_serializer", REF / "src/ignite_xdna/compiler/serializer.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    require_reference()
    S = load_serializer()
    manifest, blobs = graph_manifest(build_yolov8("n", imgsz=64), model_name="yolov8n_64")
    with tempfile.TemporaryDirectory() as d:
        w = S.IgniteModelWriter(manifest_meta=manifest, arch_id=ARCH_B200)
        for name, data, ctype in blobs:
            w.add_blob(name, data, content_type=ctype)
        size = w.write(Path(d) / "g.ignite")
        digest = hashlib.sha256((Path(d) / "g.ignite").read_bytes()).hexdigest()
    w = S.IgniteModelWriter(manifest_meta=SMALL_MANIFEST, arch_id=S.ARCH_XDNA1_PHOENIX)
    for name, data, ctype in SMALL_BLOBS:
        w.add_blob(name, data, content_type=ctype)
    w.write(HERE / "container_ref_small.ignite")
    (HERE / "container_golden.json").write_text(json.dumps(
        {"yolov8n_64": {"sha256": digest, "size": size, "model_name": "yolov8n_64"}}, indent=1) + "\n")
    print("wrote container_golden.json and container_ref_small.ignite")


if __name__ == "__main__":
    main()
