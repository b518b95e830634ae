"""Seeded synthetic YOLOv8 n/s/m graphs quantized to XINT8 with power-of-two scales.

No model files exist for this path, so the graph is built from the architecture and the
quantizer's rules, then lowered to the layer IR of ``graph.py``:

* architecture: the Ultralytics YOLOv8 layout that the reference lowers
  (``graph_ir.lower_yolov8n``, graph_ir.py:638-1185): Conv+BN folded into 3x3/1x1 convs with
  SiLU, C2f blocks (split = channel slice view, concat = ordered segment list), SPPF with three
  chained 5x5 stride-1 max-pools, FPN/PAN with nearest 2x upsample and concat, and a detect
  head of 3x3, 3x3, 1x1 convs per level emitting 64 box + 80 class channels;
* weights: kaiming-normal fp32 from the model seed, quantized per tensor to int8 at a pow2
  scale 2^-k with k = floor(log2(127 / max|w|)), ties-to-even and clipped to [-127, 127]
  (``quant/pow2.py:107-115``, ``qrange`` :16-22);
* biases: int32 at the product scale s_in * s_w;
* activation positions: max-abs over seeded calibration images in a float forward pass,
  k = floor(log2(127 / max|x|)); the input is fixed at 2^-7;
* legality rules of the quantizer's refine step (``quant/refine.py``): concat / pool / slice /
  resize operands share one position (align_concat :128-145, align_inout :147-158),
  Add operands within 7 positions (shift_read :166-175), Add output within [-7, 25] of the
  finer operand (shift_write :177-198), conv shift in [0, 16] by moving the weight position
  (shift_cut :200-210); and the SiLU epilogue's ``ysh >= 0`` (silu_sigmoid.py:146-148).

Every SiLU becomes the sigmoid-epilogue table of ``silu.fit_sigmoid`` (the reference's
``--silu-sigmoid`` graphs). The result is cached on disk by the hash of its spec.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import pickle
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np

from .graph import ConvLayer, GraphIR, PoolLayer, Segment, TensorInfo
from .silu import fit_sigmoid

HEAD_NAMES = ("p3_box", "p3_cls", "p4_box", "p4_cls", "p5_box", "p5_cls")
# YOLOv8-pose keeps the detect heads with one class and adds a keypoint branch (cv4): 17 keypoints x
# (x, y, visibility) = 51 channels per level (the reference's runtime/heads.py POSE_HEAD_NAMES)
POSE_HEAD_NAMES = HEAD_NAMES + ("p3_kpt", "p4_kpt", "p5_kpt")
POSE_KPT_CHANNELS = 51
VARIANTS = {"n": (0.33, 0.25, 1024), "s": (0.33, 0.50, 1024), "m": (0.67, 0.75, 768)}
INPUT_POS = 7
BUILD_VERSION = 1


@dataclass(frozen=True)
class ModelSpec:
    variant: str = "n"
    imgsz: int = 640
    seed: int = 0
    calib_seed: int = 1000
    n_calib: int = 8
    nc: int = 80
    reg_max: int = 16
    bias_std: float = 0.1
    task: str = "detect"      # or "pose": one class and the keypoint heads

    def key(self) -> str:
        d = asdict(self)
        if d["task"] == "detect":
            del d["task"]         # detect models keep the keys they had before pose existed
        blob = json.dumps({**d, "v": BUILD_VERSION}, sort_keys=True).encode()
        return hashlib.sha256(blob).hexdigest()[:16]


def _div8(x: float) -> int:
    return int(math.ceil(x / 8) * 8)


@dataclass
class _FConv:
    name: str
    src: List[Tuple[str, int, int, bool]]   # (tensor, channel offset, channels, up2)
    cin: int
    cout: int
    k: int
    s: int
    act: bool
    res: Optional[Tuple[str, int, int]] = None
    out: str = ""
    w: Optional[np.ndarray] = None
    b: Optional[np.ndarray] = None


@dataclass
class _FPool:
    name: str
    src: str
    out: str


@dataclass
class _FGraph:
    tensors: Dict[str, Tuple[int, int, int]] = field(default_factory=dict)   # name -> (C, H, W)
    layers: List[object] = field(default_factory=list)
    heads: Dict[str, str] = field(default_factory=dict)


class _Arch:
    """Builds the float graph in execution order."""

    def __init__(self, spec: ModelSpec):
        if spec.variant not in VARIANTS:
            raise ValueError(f"unknown YOLOv8 variant {spec.variant!r}")
        if spec.imgsz % 32:
            raise ValueError("imgsz must be a multiple of 32")
        self.spec = spec
        self.depth, self.width, self.max_ch = VARIANTS[spec.variant]
        self.g = _FGraph()
        self.g.tensors["images"] = (3, spec.imgsz, spec.imgsz)

    def ch(self, base: int) -> int:
        return _div8(min(base, self.max_ch) * self.width)

    def reps(self, n: int) -> int:
        return max(round(n * self.depth), 1)

    def conv(self, name, src, cout, k, s, act=True, res=None) -> str:
        c0, h, w = self.g.tensors[src[0][0]]
        h = h * 2 if src[0][3] else h
        w = w * 2 if src[0][3] else w
        for t, off, c, up in src:
            ct, ht, wt = self.g.tensors[t]
            ht, wt = (ht * 2, wt * 2) if up else (ht, wt)
            if (ht, wt) != (h, w) or off + c > ct:
                raise ValueError(f"{name}: inconsistent input segment {t}")
        cin = sum(c for _, _, c, _ in src)
        p = k // 2
        ho, wo = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
        out = f"{name}:out"
        self.g.tensors[out] = (cout, ho, wo)
        self.g.layers.append(_FConv(name, list(src), cin, cout, k, s, act, res, out))
        return out

    def pool(self, name, src) -> str:
        out = f"{name}:out"
        self.g.tensors[out] = self.g.tensors[src]
        self.g.layers.append(_FPool(name, src, out))
        return out

    def seg(self, t, off=0, c=None, up=False):
        return (t, off, self.g.tensors[t][0] if c is None else c, up)

    def c2f(self, idx, src, c2, n, shortcut) -> str:
        c = c2 // 2
        cv1 = self.conv(f"/model.{idx}/cv1/conv/Conv", src, 2 * c, 1, 1)
        prev = (cv1, c, c, False)
        outs = []
        for i in range(n):
            h = self.conv(f"/model.{idx}/m.{i}/cv1/conv/Conv", [prev], c, 3, 1)
            res = (prev[0], prev[1], prev[2]) if shortcut else None
            o = self.conv(f"/model.{idx}/m.{i}/cv2/conv/Conv", [self.seg(h)], c, 3, 1, res=res)
            outs.append(o)
            prev = self.seg(o)
        return self.conv(f"/model.{idx}/cv2/conv/Conv", [self.seg(cv1)] + [self.seg(o) for o in outs], c2, 1, 1)

    def build(self) -> _FGraph:
        c0, c1, c2, c3, c4 = (self.ch(b) for b in (64, 128, 256, 512, 1024))
        x = self.conv("/model.0/conv/Conv", [self.seg("images")], c0, 3, 2)
        x = self.conv("/model.1/conv/Conv", [self.seg(x)], c1, 3, 2)
        x = self.c2f(2, [self.seg(x)], c1, self.reps(3), True)
        x = self.conv("/model.3/conv/Conv", [self.seg(x)], c2, 3, 2)
        p3b = self.c2f(4, [self.seg(x)], c2, self.reps(6), True)
        x = self.conv("/model.5/conv/Conv", [self.seg(p3b)], c3, 3, 2)
        p4b = self.c2f(6, [self.seg(x)], c3, self.reps(6), True)
        x = self.conv("/model.7/conv/Conv", [self.seg(p4b)], c4, 3, 2)
        x = self.c2f(8, [self.seg(x)], c4, self.reps(3), True)
        # SPPF: cv1, three chained 5x5 pools, concat, cv2
        cs = c4 // 2
        s1 = self.conv("/model.9/cv1/conv/Conv", [self.seg(x)], cs, 1, 1)
        m1 = self.pool("/model.9/m/MaxPool", s1)
        m2 = self.pool("/model.9/m_1/MaxPool", m1)
        m3 = self.pool("/model.9/m_2/MaxPool", m2)
        p5b = self.conv("/model.9/cv2/conv/Conv", [self.seg(t) for t in (s1, m1, m2, m3)], c4, 1, 1)
        n3 = self.reps(3)
        h12 = self.c2f(12, [self.seg(p5b, up=True), self.seg(p4b)], c3, n3, False)
        p3 = self.c2f(15, [self.seg(h12, up=True), self.seg(p3b)], c2, n3, False)
        x = self.conv("/model.16/conv/Conv", [self.seg(p3)], c2, 3, 2)
        p4 = self.c2f(18, [self.seg(x), self.seg(h12)], c3, n3, False)
        x = self.conv("/model.19/conv/Conv", [self.seg(p4)], c3, 3, 2)
        p5 = self.c2f(21, [self.seg(x), self.seg(p5b)], c4, n3, False)
        nc, rm = self.spec.nc, self.spec.reg_max
        cb = max(16, c2 // 4, rm * 4)
        cc = max(c2, min(nc, 100))
        for i, feat in enumerate((p3, p4, p5)):
            b = self.conv(f"/model.22/cv2.{i}/cv2.{i}.0/conv/Conv", [self.seg(feat)], cb, 3, 1)
            b = self.conv(f"/model.22/cv2.{i}/cv2.{i}.1/conv/Conv", [self.seg(b)], cb, 3, 1)
            b = self.conv(f"/model.22/cv2.{i}/cv2.{i}.2/Conv", [self.seg(b)], 4 * rm, 1, 1, act=False)
            c = self.conv(f"/model.22/cv3.{i}/cv3.{i}.0/conv/Conv", [self.seg(feat)], cc, 3, 1)
            c = self.conv(f"/model.22/cv3.{i}/cv3.{i}.1/conv/Conv", [self.seg(c)], cc, 3, 1)
            c = self.conv(f"/model.22/cv3.{i}/cv3.{i}.2/Conv", [self.seg(c)], nc, 1, 1, act=False)
            self.g.heads[f"p{i + 3}_box"] = b
            self.g.heads[f"p{i + 3}_cls"] = c
            if self.spec.task == "pose":
                ck = max(c2 // 4, POSE_KPT_CHANNELS)
                k = self.conv(f"/model.22/cv4.{i}/cv4.{i}.0/conv/Conv", [self.seg(feat)], ck, 3, 1)
                k = self.conv(f"/model.22/cv4.{i}/cv4.{i}.1/conv/Conv", [self.seg(k)], ck, 3, 1)
                k = self.conv(f"/model.22/cv4.{i}/cv4.{i}.2/Conv", [self.seg(k)], POSE_KPT_CHANNELS, 1, 1, act=False)
                self.g.heads[f"p{i + 3}_kpt"] = k
        return self.g


def _init_weights(g: _FGraph, spec: ModelSpec) -> None:
    rng = np.random.default_rng(spec.seed)
    for L in g.layers:
        if isinstance(L, _FConv):
            fan_in = L.cin * L.k * L.k
            L.w = (rng.standard_normal((L.cout, L.cin, L.k, L.k), dtype=np.float32)
                   * np.float32(math.sqrt(2.0 / fan_in)))
            L.b = rng.standard_normal(L.cout, dtype=np.float32) * np.float32(spec.bias_std)


def calibration_images(spec: ModelSpec) -> np.ndarray:
    """uint8 [n, 3, H, W] uniform over [0, 255], image i from seed calib_seed + i."""
    return np.stack([np.random.default_rng(spec.calib_seed + i).integers(
        0, 256, size=(3, spec.imgsz, spec.imgsz), dtype=np.uint8) for i in range(spec.n_calib)])


def _calibrate(g: _FGraph, spec: ModelSpec) -> Dict[str, float]:
    """Max-abs of every float tensor: '<conv>:pre' (linear), '<conv>:act' (after SiLU), '<t>' (stored)."""
    import torch
    import torch.nn.functional as F
    amax: Dict[str, float] = {}
    imgs = calibration_images(spec)
    with torch.no_grad():
        for i in range(imgs.shape[0]):
            vals: Dict[str, torch.Tensor] = {"images": torch.from_numpy(imgs[i:i + 1].astype(np.float32) / 255.0)}
            for L in g.layers:
                if isinstance(L, _FConv):
                    parts = []
                    for t, off, c, up in L.src:
                        v = vals[t][:, off:off + c]
                        if up:
                            v = F.interpolate(v, scale_factor=2, mode="nearest")
                        parts.append(v)
                    x = torch.cat(parts, dim=1) if len(parts) > 1 else parts[0]
                    pre = F.conv2d(x, torch.from_numpy(L.w), torch.from_numpy(L.b), stride=L.s, padding=L.k // 2)
                    keys = {f"{L.name}:pre": pre}
                    y = pre
                    if L.act:
                        y = F.silu(pre)
                        keys[f"{L.name}:act"] = y
                    if L.res is not None:
                        t, off, c = L.res
                        y = y + vals[t][:, off:off + c]
                    vals[L.out] = y
                    keys[L.out] = y
                    for k, v in keys.items():
                        amax[k] = max(amax.get(k, 0.0), float(v.abs().max()))
                else:
                    y = F.max_pool2d(vals[L.src], 5, 1, 2)
                    vals[L.out] = y
                    amax[L.out] = max(amax.get(L.out, 0.0), float(y.abs().max()))
    return amax


def _pos_of(amax: float) -> int:
    if not amax > 0:
        return INPUT_POS
    return int(math.floor(math.log2(127.0 / amax)))


def _quantize_pow2(x: np.ndarray, pos: int) -> np.ndarray:
    """float32 divide by 2^-pos, ties to even, clip to the symmetric int8 range [-127, 127]."""
    scale = np.float32(np.ldexp(1.0, -pos))
    return np.clip(np.rint(x.astype(np.float32) / scale), -127, 127).astype(np.int8)


class _Groups:
    def __init__(self):
        self.parent: Dict[str, str] = {}

    def find(self, a):
        self.parent.setdefault(a, a)
        while self.parent[a] != a:
            self.parent[a] = self.parent[self.parent[a]]
            a = self.parent[a]
        return a

    def union(self, a, b):
        self.parent[self.find(a)] = self.find(b)

    def members(self):
        out: Dict[str, List[str]] = {}
        for a in list(self.parent):
            out.setdefault(self.find(a), []).append(a)
        return list(out.values())


def _refine(g: _FGraph, pos: Dict[str, int]) -> None:
    groups = _Groups()
    for L in g.layers:
        if isinstance(L, _FConv):
            for t, _, _, _ in L.src:
                groups.union(t, L.src[0][0])
        else:
            groups.union(L.src, L.out)
    members = groups.members()
    for _ in range(200):
        changed = False
        for m in members:
            lo = min(pos[t] for t in m)
            for t in m:
                if pos[t] != lo:
                    pos[t], changed = lo, True
        for L in g.layers:
            if not isinstance(L, _FConv):
                continue
            if L.res is not None:
                a, r, o = f"{L.name}:act", L.res[0], L.out
                if max(pos[a], pos[r]) - min(pos[a], pos[r]) > 7:
                    hi = a if pos[a] > pos[r] else r
                    pos[hi] = min(pos[a], pos[r]) + 7
                    changed = True
                low = min(pos[a], pos[r])
                sw = low - pos[o]
                if sw > 25 or sw < -7:
                    pos[o] = low - min(max(sw, -7), 25)
                    changed = True
            if L.act:
                a = f"{L.name}:act"
                if pos[a] > pos[f"{L.name}:pre"] + 7:
                    pos[a] = pos[f"{L.name}:pre"] + 7
                    changed = True
        if not changed:
            return
    raise RuntimeError("quantizer position rules did not converge")


def _build(spec: ModelSpec) -> GraphIR:
    g = _Arch(spec).build()
    _init_weights(g, spec)
    amax = _calibrate(g, spec)
    pos = {k: _pos_of(v) for k, v in amax.items()}
    pos["images"] = INPUT_POS
    for L in g.layers:
        if isinstance(L, _FConv) and L.act and L.res is None:
            pos[f"{L.name}:act"] = pos[L.out]
    _refine(g, pos)
    for L in g.layers:   # without a residual the activation is the stored tensor
        if isinstance(L, _FConv) and L.act and L.res is None:
            pos[f"{L.name}:act"] = pos[L.out]
    tensors: Dict[str, TensorInfo] = {}
    c, h, w = g.tensors["images"]
    tensors["images"] = TensorInfo("images", c, h, w, 2.0 ** -INPUT_POS, producer="input")
    layers: List[object] = []
    for L in g.layers:
        if isinstance(L, _FPool):
            c, h, w = g.tensors[L.out]
            tensors[L.out] = TensorInfo(L.out, c, h, w, 2.0 ** -pos[L.out], producer=L.name)
            layers.append(PoolLayer(L.name, len(layers), Segment(L.src, 0, c // 8), L.out))
            continue
        p_in = pos[L.src[0][0]]
        p_pre = pos[f"{L.name}:pre"]
        p_w = _pos_of(float(np.abs(L.w).max()))
        sc = p_w + p_in - p_pre
        if sc < 0 or sc > 16:            # shift_cut: move the weight position
            p_w = min(max(sc, 0), 16) + p_pre - p_in
        wq = _quantize_pow2(L.w, p_w)
        bscale = 2.0 ** -(p_in + p_w)
        bq = np.clip(np.rint(L.b.astype(np.float64) / bscale), -(2 ** 31), 2 ** 31 - 1).astype(np.int32)
        segs = [Segment(t, off // 8, (cc + 7) // 8, up) for t, off, cc, up in L.src]
        layer = ConvLayer(name=L.name, index=len(layers), inputs=segs, in_scale=2.0 ** -p_in, k=L.k, stride=L.s,
                          pad=L.k // 2, weights=wq, bias_q=bq, bias_scale=bscale, weight_scale=2.0 ** -p_w,
                          conv_scale=2.0 ** -p_pre, output=L.out)
        if L.act:
            p_act = pos[f"{L.name}:act"]
            layer.act = "silu_sigmoid"
            layer.act_scale = 2.0 ** -p_act
            layer.sigmoid = fit_sigmoid(2.0 ** -p_pre, 2.0 ** -p_act)
            out_pos = p_act
        else:
            out_pos = p_pre
        if L.res is not None:
            t, off, cc = L.res
            p_res, p_add = pos[t], pos[L.out]
            p_fine = max(out_pos, p_res, p_add)     # finest of the three scales
            layer.residual = Segment(t, off // 8, cc // 8)
            layer.residual_lsh_main = p_fine - out_pos
            layer.residual_lsh_res = p_fine - p_res
            layer.residual_shift = p_fine - p_add
            out_pos = p_add
        c, h, w = g.tensors[L.out]
        tensors[L.out] = TensorInfo(L.out, c, h, w, 2.0 ** -out_pos, producer=L.name)
        if not 0 <= layer.shift_out <= 16:
            raise ValueError(f"{L.name}: shift {layer.shift_out} outside [0, 16]")
        acc_bound = int(np.abs(layer.bias_int8_domain()).max()) + L.cin * L.k * L.k * 127 * 128
        if acc_bound >= 2 ** 31 or int(np.abs(layer.bias_acc()).max()) >= 2 ** 31:
            raise ValueError(f"{L.name}: accumulator may leave int32")
        layers.append(layer)
    names = POSE_HEAD_NAMES if spec.task == "pose" else HEAD_NAMES
    outputs = [(name, g.heads[name]) for name in names]
    return GraphIR(tensors=tensors, layers=layers, input="images", outputs=outputs, silu_sigmoid=True,
                   task=spec.task, spec={**asdict(spec), "key": spec.key()})


def default_cache_dir() -> Path:
    env = os.environ.get("IXB_MODEL_CACHE")
    if env:
        return Path(env)
    return Path(__file__).resolve().parent.parent / "build" / "models"


def build_yolov8(variant: str = "n", imgsz: int = 640, seed: int = 0, cache: bool = True, **kw) -> GraphIR:
    """The quantized synthetic YOLOv8 graph for ``variant`` in {"n", "s", "m"}; ``task="pose"``
    builds YOLOv8-pose (one class, keypoint heads)."""
    if kw.get("task") == "pose":
        kw.setdefault("nc", 1)
    spec = ModelSpec(variant=variant, imgsz=imgsz, seed=seed, **kw)
    tag = "-pose" if spec.task == "pose" else ""
    path = default_cache_dir() / f"yolov8{variant}{tag}_{imgsz}_{spec.key()}.pkl"
    if cache and path.exists():
        with open(path, "rb") as f:
            return pickle.load(f)
    ir = _build(spec)
    if cache:
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        with open(tmp, "wb") as f:
            pickle.dump(ir, f)
        os.replace(tmp, path)
    return ir


def random_images(batch: int, imgsz: int = 640, seed: int = 0) -> np.ndarray:
    """uint8 [batch, 3, imgsz, imgsz] uniform over [0, 255] from one seed."""
    return np.random.default_rng(seed).integers(0, 256, size=(batch, 3, imgsz, imgsz), dtype=np.uint8)
