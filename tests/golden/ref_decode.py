"""ctypes binding of the reference's own CPU decode, pipelines/decode_native.c yolo_decode_int8,
built from the reference's sources by oracle/build_ref.sh into oracle/_ref/decode_native.so.
Test infrastructure: it is the checker for the GPU decode, never part of the engine."""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Optional

import numpy as np

REF_SO = Path(__file__).resolve().parents[2] / "oracle" / "_ref" / "decode_native.so"


class _Head(C.Structure):   # yolo_head_t (decode_native.c:58-69)
    _fields_ = [("box", C.c_void_p), ("cls", C.c_void_p), ("cls_max", C.c_void_p), ("dfl_exp", C.c_void_p),
                ("box_val", C.c_void_p), ("sigmoid", C.c_void_p), ("sigmoid_low", C.c_void_p),
                ("q_threshold", C.c_double), ("anchors", C.c_int32), ("anchor_offset", C.c_int32)]


class _Decode(C.Structure):  # yolo_decode_t (decode_native.c:71-80)
    _fields_ = [("head", _Head * 3), ("anchor_x", C.c_void_p), ("anchor_y", C.c_void_p), ("strides", C.c_void_p),
                ("reg_max", C.c_int32), ("num_classes", C.c_int32), ("conf", C.c_float), ("iou", C.c_float)]


def load() -> Optional[C.CDLL]:
    if not REF_SO.exists():
        return None
    lib = C.CDLL(str(REF_SO))
    lib.yolo_decode_int8.argtypes = [C.c_void_p, C.c_float, C.c_float, C.c_float, C.c_int32,
                                     C.c_void_p, C.c_void_p, C.c_void_p]
    lib.yolo_decode_int8.restype = C.c_int
    return lib


def decode(lib, egress_image: np.ndarray, layout, tables, anchors, conf: float, iou: float,
           letterbox=(0.0, 0.0, 1.0), num_classes: int = 80):
    """Run the reference decode on one image's int8 egress. tables: per head (dfl, sigmoid, low, q_thr)."""
    d = _Decode()
    keep = []
    off = 0
    for h, (bname, cname) in enumerate((("p3_box", "p3_cls"), ("p4_box", "p4_cls"), ("p5_box", "p5_cls"))):
        bs, cs = layout.spec(bname), layout.spec(cname)
        n = bs.shape[1] * bs.shape[2]
        box = np.ascontiguousarray(egress_image[bs.offset:bs.end])
        cls = np.ascontiguousarray(egress_image[cs.offset:cs.end])
        dfl, sig, low, qt = tables[h]
        keep += [box, cls, dfl, sig, low]
        hd = d.head[h]
        hd.box, hd.cls, hd.cls_max = box.ctypes.data, cls.ctypes.data, None
        hd.dfl_exp, hd.box_val, hd.sigmoid = dfl.ctypes.data, None, sig.ctypes.data
        hd.sigmoid_low = low.ctypes.data if low is not None else None
        hd.q_threshold, hd.anchors, hd.anchor_offset = qt, n, off
        off += n
    ax, ay, st = anchors
    d.anchor_x, d.anchor_y, d.strides = ax.ctypes.data, ay.ctypes.data, st.ctypes.data
    d.reg_max, d.num_classes = 16, num_classes
    d.conf, d.iou = float(np.float32(conf)), float(np.float32(iou))
    cap = off
    ob = np.zeros(4 * cap, np.float32)
    osc = np.zeros(cap, np.float32)
    ocl = np.zeros(cap, np.int32)
    n = lib.yolo_decode_int8(C.addressof(d), float(letterbox[0]), float(letterbox[1]), float(letterbox[2]), cap,
                             ob.ctypes.data, osc.ctypes.data, ocl.ctypes.data)
    if n < 0:
        raise RuntimeError(f"reference decode failed ({n})")
    return ob[:4 * n].reshape(n, 4), osc[:n], ocl[:n]
