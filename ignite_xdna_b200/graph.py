"""Layer IR of a quantized XINT8 YOLOv8 graph.

The record types carry the same fields, with the same meaning, as the reference's
``src/ignite_xdna/compiler/graph_ir.py`` (``TensorInfo`` :51-67, ``Segment`` :69-74,
``ConvLayer`` :85-134, ``PoolLayer`` :222-229, ``GraphIR`` :262-273), so a graph built here
can be handed to the reference's integer reference unchanged, and the device plan
(``plan.py``) reads exactly what the reference's compiler reads.

Activations are uint8 with zero point 128 and a power-of-two scale in the reference.
The device stores the same values as int8 ``t = q - 128``; ``plan.py`` and the kernels
use the un-folded accumulator bias ``bias_q << e`` for that domain, while
``ConvLayer.bias_acc`` gives the reference's folded uint8-domain bias (graph_ir.py:126-134).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

ZP = 128


def log2_exact(scale: float) -> int:
    """Exponent of a power-of-two scale; refuses anything else (graph_ir.py:44-48)."""
    e = math.log2(scale)
    if abs(e - round(e)) > 1e-9:
        raise ValueError(f"scale {scale} is not a power of two")
    return int(round(e))


@dataclass
class TensorInfo:
    """One physical activation tensor (uint8, zero point 128 in the reference's terms)."""
    name: str
    channels: int
    height: int
    width: int
    scale: float
    zero_point: int = ZP
    producer: str = ""

    @property
    def blocks(self) -> int:
        return (self.channels + 7) // 8


@dataclass
class Segment:
    """A channel-block view of a tensor: blocks of 8 channels, optionally nearest-2x upsampled."""
    tensor: str
    block_offset: int
    blocks: int
    up2: bool = False


@dataclass
class SigmoidFit:
    """The four-line sigmoid SiLU epilogue of one (s1, s2) pair and its 256-entry table.

    ``table`` is indexed by the uint8 linear conv output q1 and holds the uint8 activation."""
    lines: Tuple[Tuple[int, int], ...]
    s: int
    ysh: int
    table: np.ndarray
    max_error: int
    mean_error: float


@dataclass
class ConvLayer:
    name: str
    index: int
    inputs: List[Segment]
    in_scale: float
    k: int
    stride: int
    pad: int
    weights: np.ndarray          # int8 [Cout][Cin][k][k]
    bias_q: np.ndarray           # int32 [Cout] at bias_scale
    bias_scale: float
    weight_scale: float
    conv_scale: float            # scale of the linear conv output (s1)
    output: str
    act: Optional[str] = None    # "silu_sigmoid" or None (a linear head conv)
    sigmoid: Optional[SigmoidFit] = None
    residual: Optional[Segment] = None
    residual_shift: int = 0
    residual_lsh_main: int = 0
    residual_lsh_res: Optional[int] = None
    act_scale: Optional[float] = None

    @property
    def cin(self) -> int:
        return int(self.weights.shape[1])

    @property
    def cout(self) -> int:
        return int(self.weights.shape[0])

    @property
    def shift_out(self) -> int:
        """SRS shift: -log2 s_in - log2 s_w + log2 s1 (graph_ir.py:122-124)."""
        return -log2_exact(self.in_scale) - log2_exact(self.weight_scale) + log2_exact(self.conv_scale)

    @property
    def bias_exp(self) -> int:
        e = log2_exact(self.bias_scale / (self.in_scale * self.weight_scale))
        if e < 0:
            raise ValueError(f"{self.name}: bias scale ratio is fractional")
        return e

    def bias_int8_domain(self) -> np.ndarray:
        """Accumulator bias for int8 activations t = q - 128: bias_q << e."""
        return self.bias_q.astype(np.int64) << self.bias_exp

    def bias_acc(self) -> np.ndarray:
        """The reference's uint8-domain bias: (bias_q << e) - 128 * sum(w) + (128 << shift)."""
        wsum = self.weights.astype(np.int64).sum(axis=(1, 2, 3))
        return (self.bias_int8_domain() - ZP * wsum + (ZP << self.shift_out)).astype(np.int64)

    def lut_t(self) -> np.ndarray:
        """Activation as an int8 table over t1 = q1 - 128 (identity for a linear layer)."""
        if self.sigmoid is None:
            return np.arange(-128, 128, dtype=np.int64).astype(np.int8)
        return (self.sigmoid.table.astype(np.int64) - ZP).astype(np.int8)


@dataclass
class PoolLayer:
    name: str
    index: int
    input: Segment
    output: str
    k: int = 5
    pad: int = 2


@dataclass
class GraphIR:
    tensors: Dict[str, TensorInfo]
    layers: List[object]
    input: str
    outputs: List[Tuple[str, str]]     # (head name, physical tensor)
    silu_sigmoid: bool = True
    task: str = "detect"
    spec: Dict[str, object] = field(default_factory=dict)

    def conv_layers(self) -> List[ConvLayer]:
        return [L for L in self.layers if isinstance(L, ConvLayer)]

    def pool_layers(self) -> List[PoolLayer]:
        return [L for L in self.layers if isinstance(L, PoolLayer)]

    def macs_per_image(self) -> int:
        total = 0
        for L in self.conv_layers():
            t = self.tensors[L.output]
            total += t.height * t.width * L.cout * L.cin * L.k * L.k
        return total
