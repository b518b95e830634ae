"""The seeded synthetic YOLOv8 graphs: structure, quantizer rules, determinism."""
import json

import numpy as np
import pytest

from ignite_xdna_b200 import build_yolov8
from ignite_xdna_b200.graph import log2_exact

import make_golden


@pytest.mark.parametrize("variant,convs", [("n", 63), ("s", 63), ("m", 83)])
def test_structure_counts(variant, convs):
    """Counts of the reference's structural test (tests/test_graph_engine_offline.py:37-44)."""
    ir = build_yolov8(variant)
    cl = ir.conv_layers()
    assert len(cl) == convs
    assert len(ir.pool_layers()) == 3
    assert sum(L.act is not None for L in cl) == convs - 6
    assert sum(s.up2 for L in cl for s in L.inputs) == 2
    assert len(ir.outputs) == 6


def test_yolov8n_macs_and_residuals():
    ir = build_yolov8("n")
    assert ir.macs_per_image() == 4_371_456_000
    assert sum(L.residual is not None for L in ir.conv_layers()) == 6


@pytest.mark.parametrize("variant", ["n", "s", "m"])
def test_quantizer_rules(variant):
    """shift_out >= 0 and |bias_acc| < 2^31 (tests/test_graph_engine_offline.py:46-53), pow2 scales,
    concat operands at one scale, SiLU ysh >= 0."""
    ir = build_yolov8(variant)
    for L in ir.conv_layers():
        assert 0 <= L.shift_out <= 16
        assert int(np.abs(L.bias_acc()).max()) < 2 ** 31
        assert L.weights.min() >= -127 and L.weights.max() <= 127
        scales = {ir.tensors[s.tensor].scale for s in L.inputs}
        assert len(scales) == 1 and abs(scales.pop() - L.in_scale) < 1e-15
        if L.sigmoid is not None:
            assert L.sigmoid.ysh >= 0
        for v in (L.in_scale, L.weight_scale, L.conv_scale):
            log2_exact(v)
    for P in ir.pool_layers():
        assert ir.tensors[P.input.tensor].scale == ir.tensors[P.output].scale


@pytest.mark.parametrize("variant", ["n", "s", "m"])
def test_builder_reproduces_golden_model(golden_dir, variant):
    """The model the fixtures were made from is rebuilt bit for bit (seeded weights, calibration)."""
    h = json.loads((golden_dir / "graph_hashes.json").read_text())[f"yolov8{variant}"]
    ir = build_yolov8(variant, cache=False)
    fp = make_golden.fingerprint(ir)
    assert fp["model"] == h["fingerprint"]["model"]
