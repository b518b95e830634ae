"""GPU detect decode + NMS for the engine's heads: the tables and anchor grid, and the call.

The device kernel (``csrc/ixb_decode.cuh``, ``ixb_decode_yolo``) reproduces the reference's
``pipelines/decode_native.c`` ``yolo_decode_int8`` bit for bit. It reads every exp from tables
that must hold the same bits as the reference's, so they are built here with the same numpy
expressions as ``pipelines/decode_native.py`` (``_dequantized_logits`` :121-122, ``dfl_exp_table``
:125-131, ``sigmoid_table`` :134-139, ``sigmoid_low_table`` :142-151, the prune threshold
:206-208, :232-233) and the anchor grid of ``pipelines/yolo_pipeline.py`` (:191-203).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib as L

STRIDES = (8, 16, 32)
REG_MAX = 16
HEAD_PAIRS = (("p3_box", "p3_cls"), ("p4_box", "p4_cls"), ("p5_box", "p5_cls"))


def dequantized_logits(scale: float, zero_point: int) -> np.ndarray:
    return (np.arange(-128, 128).astype(np.float32) - np.float32(zero_point)) * np.float32(scale)


def dfl_exp_table(scale: float, zero_point: int) -> np.ndarray:
    """float32 [256][256]: exp(v(q) - v(q_max)) at [q_max + 128][q + 128]."""
    v = dequantized_logits(scale, zero_point)
    with np.errstate(over="ignore"):
        t = np.exp(v[None, :] - v[:, None])
    return np.ascontiguousarray(t, dtype=np.float32)


def sigmoid_table(scale: float, zero_point: int) -> np.ndarray:
    """float32 [256]: 1 / (1 + exp(-v(q))) at [q + 128]."""
    v = dequantized_logits(scale, zero_point)
    with np.errstate(over="ignore"):
        t = 1.0 / (1.0 + np.exp(-v))
    return np.ascontiguousarray(t, dtype=np.float32)


def sigmoid_low_table(sig: np.ndarray) -> Optional[np.ndarray]:
    """int32 [256]: the smallest q whose sigmoid equals that of q, or None if the table is not monotone."""
    if not np.all(sig[1:] >= sig[:-1]):
        return None
    return np.ascontiguousarray(np.searchsorted(sig, sig, side="left") - 128, dtype=np.int32)


def q_threshold(conf: float, scale: float, zero_point: int) -> float:
    c = min(max(float(conf), 1e-12), 1.0 - 1e-12)
    return float(np.log(c / (1.0 - c)) / float(scale) + int(zero_point))


def anchor_grid(imgsz: int, strides: Sequence[int] = STRIDES) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Anchor centres x, y and the stride per anchor, float32 [sum g^2], level by level."""
    xs, ys, ss = [], [], []
    for s in strides:
        g = imgsz // s
        c = np.arange(g, dtype=np.float32) + 0.5
        yy, xx = np.meshgrid(c, c, indexing="ij")
        xs.append(xx.ravel())
        ys.append(yy.ravel())
        ss.append(np.full(g * g, float(s), np.float32))
    return (np.concatenate(xs).astype(np.float32), np.concatenate(ys).astype(np.float32),
            np.concatenate(ss).astype(np.float32))


class DecodeHead(C.Structure):
    _fields_ = [("box_offset", C.c_uint64), ("cls_offset", C.c_uint64), ("dfl_exp", C.c_void_p),
                ("sigmoid", C.c_void_p), ("sigmoid_low", C.c_void_p), ("q_threshold", C.c_double),
                ("anchors", C.c_int32), ("anchor_offset", C.c_int32)]


class DecodeDesc(C.Structure):
    _fields_ = [("head", DecodeHead * 3), ("anchor_x", C.c_void_p), ("anchor_y", C.c_void_p),
                ("strides", C.c_void_p), ("reg_max", C.c_int32), ("num_classes", C.c_int32),
                ("conf", C.c_float), ("iou", C.c_float)]


class DetectConfig(C.Structure):
    _fields_ = [("decode", DecodeDesc), ("cls_scale", C.c_float * 3), ("cls_zero_point", C.c_int32 * 3),
                ("capacity", C.c_int32)]


@dataclass
class Detections:
    boxes: np.ndarray      # float32 [n, 4]: x0, y0, w, h in source-image pixels
    scores: np.ndarray     # float32 [n]
    classes: np.ndarray    # int32 [n]


class GpuDecoder:
    """Decode + NMS of a session's device egress: tables on the device once per (scales, thresholds)."""

    def __init__(self, layout, imgsz: int, device, num_classes: int = 80, conf: float = 0.25, iou: float = 0.50):
        import torch
        self.lib = L.load()
        self.layout = layout
        self.device = device
        self.num_classes = int(num_classes)
        self.conf = float(conf)
        self.iou = float(iou)
        ax, ay, st = anchor_grid(imgsz)
        self.total_anchors = ax.size
        self._keep = [torch.from_numpy(a).to(device) for a in (ax, ay, st)]
        d = DecodeDesc()
        off = 0
        for h, (bname, cname) in enumerate(HEAD_PAIRS):
            bs, cs = layout.spec(bname), layout.spec(cname)
            n = bs.shape[1] * bs.shape[2]
            if bs.shape[0] != 4 * REG_MAX or cs.shape[0] != self.num_classes or cs.shape[1] * cs.shape[2] != n:
                raise ValueError(f"head pair {bname}/{cname} does not match the decode layout")
            dfl = torch.from_numpy(dfl_exp_table(bs.scale, bs.zero_point)).to(device)
            sig_np = sigmoid_table(cs.scale, cs.zero_point)
            sig = torch.from_numpy(sig_np).to(device)
            low_np = sigmoid_low_table(sig_np)
            low = torch.from_numpy(low_np).to(device) if low_np is not None else None
            self._keep += [dfl, sig] + ([low] if low is not None else [])
            hd = d.head[h]
            hd.box_offset, hd.cls_offset = bs.offset, cs.offset
            hd.dfl_exp, hd.sigmoid = dfl.data_ptr(), sig.data_ptr()
            hd.sigmoid_low = low.data_ptr() if low is not None else None
            hd.q_threshold = q_threshold(self.conf, cs.scale, cs.zero_point)
            hd.anchors, hd.anchor_offset = n, off
            off += n
        d.anchor_x, d.anchor_y, d.strides = (t.data_ptr() for t in self._keep[:3])
        d.reg_max, d.num_classes = REG_MAX, self.num_classes
        d.conf, d.iou = float(np.float32(self.conf)), float(np.float32(self.iou))
        self.desc = d
        self.cls_quant = [(layout.spec(c).scale, layout.spec(c).zero_point) for _, c in HEAD_PAIRS]

    def config(self, capacity: int) -> DetectConfig:
        """The session-level detection stage's configuration (ixb_session_set_detect)."""
        c = DetectConfig()
        c.decode = self.desc
        for h, (sc, zp) in enumerate(self.cls_quant):
            c.cls_scale[h], c.cls_zero_point[h] = float(sc), int(zp)
        c.capacity = int(capacity)
        return c

    def __call__(self, egress_dev, batch: int, letterbox=None, capacity: Optional[int] = None,
                 stream: Optional[int] = None) -> List[Detections]:
        """egress_dev: uint8/int8 CUDA tensor holding `batch` images' egress back to back."""
        import torch
        cap = int(capacity if capacity is not None else self.total_anchors)
        if letterbox is None:
            lb = torch.zeros((batch, 3), dtype=torch.float32, device=self.device)
            lb[:, 2] = 1.0
        else:
            lb = torch.as_tensor(np.asarray(letterbox, dtype=np.float32).reshape(batch, 3), device=self.device)
        boxes = torch.empty((batch, cap, 4), dtype=torch.float32, device=self.device)
        scores = torch.empty((batch, cap), dtype=torch.float32, device=self.device)
        classes = torch.empty((batch, cap), dtype=torch.int32, device=self.device)
        counts = torch.empty(batch, dtype=torch.int32, device=self.device)
        L.check(self.lib.ixb_decode_yolo(C.byref(self.desc), C.c_void_p(egress_dev.data_ptr()), int(batch),
                                         self.layout.image_bytes, C.c_void_p(lb.data_ptr()), cap,
                                         C.c_void_p(boxes.data_ptr()), C.c_void_p(scores.data_ptr()),
                                         C.c_void_p(classes.data_ptr()), C.c_void_p(counts.data_ptr()),
                                         C.c_void_p(stream) if stream else None))
        n = counts.cpu().numpy()
        b, s, c = boxes.cpu().numpy(), scores.cpu().numpy(), classes.cpu().numpy()
        out = []
        for i in range(batch):
            if n[i] < 0:
                raise RuntimeError(f"image {i}: more than {cap} detections survive NMS")
            out.append(Detections(b[i, :n[i]].copy(), s[i, :n[i]].copy(), c[i, :n[i]].copy()))
        return out


def dense_heads(layout, imgsz: int, strides: Sequence[int] = STRIDES):
    """ixb_dense_head[3] of a session's egress: each level's box and class heads, their scales and
    zero points, grid and stride."""
    heads = (L.DenseHead * 3)()
    for h, ((bname, cname), s) in enumerate(zip(HEAD_PAIRS, strides)):
        bs, cs = layout.spec(bname), layout.spec(cname)
        if bs.shape[0] != 4 * REG_MAX or bs.shape[1] != bs.shape[2] or bs.shape[1] * s != imgsz:
            raise ValueError(f"head {bname} does not match a {imgsz}x{imgsz} stride-{s} level")
        d = heads[h]
        d.box_offset, d.cls_offset = bs.offset, cs.offset
        d.box_scale, d.box_zero_point = float(bs.scale), int(bs.zero_point)
        d.cls_scale, d.cls_zero_point = float(cs.scale), int(cs.zero_point)
        d.grid, d.stride = bs.shape[1], float(s)
    return heads
