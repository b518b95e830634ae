"""Detect-head egress layout: the six raw int8 heads as NCHW views of one egress buffer.

Same contract as the reference's ``src/ignite_xdna/runtime/heads.py`` (``HeadSpec`` :47-76,
``DetectHeadLayout`` :79-140, ``HeadStatus`` :143-150): per head a byte offset, a 4-D shape,
a dequantisation scale and zero point 0; unpacking is zero-copy. Here the layout is produced
by the engine's own plan (heads back to back in the graph's output order per image: the six
detect heads ``HEAD_NAMES``, then for a pose graph the three keypoint heads) and carries a
leading batch dimension.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Mapping, Optional, Tuple

import numpy as np

from .yolov8 import HEAD_NAMES  # noqa: F401  (re-exported: the detect heads' names)


@dataclass(frozen=True)
class HeadSpec:
    name: str
    shape: Tuple[int, ...]        # (C, H, W) per image
    offset: int                   # bytes into one image's egress
    scale: float
    zero_point: int = 0

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape))

    @property
    def end(self) -> int:
        return self.offset + self.nbytes


@dataclass(frozen=True)
class DetectHeadLayout:
    heads: Tuple[HeadSpec, ...]
    image_bytes: int

    def spec(self, name: str) -> HeadSpec:
        for h in self.heads:
            if h.name == name:
                return h
        raise KeyError(name)

    def scales(self) -> Dict[str, Tuple[float, int]]:
        return {h.name: (h.scale, h.zero_point) for h in self.heads}

    def unpack(self, raw: np.ndarray) -> Dict[str, np.ndarray]:
        """int8 [B, image_bytes] (or one flat image) -> {head: int8 [B, C, H, W]} views, no copy."""
        a = np.asarray(raw)
        if a.dtype != np.int8:
            raise TypeError(f"egress must be int8, got {a.dtype}")
        a = a.reshape(-1, self.image_bytes)
        return {h.name: a[:, h.offset:h.end].reshape((a.shape[0],) + h.shape) for h in self.heads}

    def dequantize(self, views: Mapping[str, np.ndarray]) -> Dict[str, np.ndarray]:
        return {h.name: (views[h.name].astype(np.float32) - np.float32(h.zero_point)) * np.float32(h.scale)
                for h in self.heads}


@dataclass(frozen=True)
class HeadStatus:
    present: bool
    reason: str
    layout: Optional[DetectHeadLayout] = None


def layout_from_plan(dp) -> DetectHeadLayout:
    ir = dp.ir
    tensor_of = dict(ir.outputs)
    specs = []
    for name, _ in ir.outputs:
        t = ir.tensors[tensor_of[name]]
        specs.append(HeadSpec(name, (t.channels, t.height, t.width), dp.head_offsets[name], t.scale, 0))
    return DetectHeadLayout(tuple(specs), dp.egress_image_bytes)
