"""Conv SRS shifts outside [0, 16], on a B200 through the C ABI.

The engine's epilogue rounds through the float unit, exact for shifts up to 16 and for left
shifts; a layer whose shift is larger takes the generic drain, which first reduces the
accumulator by shift - 16 with a sticky bit. These graphs are the seeded YOLOv8n at 64x64 with
one SiLU conv and one linear head conv re-scaled so their SRS shift lands outside [0, 16]
(their output scale multiplied by a power of two, activation table kept), so the whole network
downstream sees the changed values; every tensor must still equal the oracle byte for byte.
"""
import copy

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import build_yolov8, random_images
from ignite_xdna_b200.session import GraphSession

pytestmark = pytest.mark.gpu


def rescaled(shift_silu: int, shift_head: int):
    """The 64x64 YOLOv8n graph with one mid-network SiLU conv and the P3 box head's last conv
    given these SRS shifts (conv_scale times a power of two)."""
    ir = copy.deepcopy(build_yolov8("n", imgsz=64))
    convs = ir.conv_layers()
    silu = next(L for L in convs if L.name.startswith("/model.4/m.0/cv1"))
    head = next(L for L in convs if L.sigmoid is None and L.output == dict(ir.outputs)["p3_box"])
    for L, s in ((silu, shift_silu), (head, shift_head)):
        L.conv_scale *= 2.0 ** (s - L.shift_out)
        assert L.shift_out == s
    if shift_head != head.shift_out:
        raise AssertionError("head rescale failed")
    # a linear head's output scale is its conv scale: keep the head tensor's scale in step
    ir.tensors[head.output].scale = head.conv_scale
    return ir


@pytest.mark.parametrize("shift_silu,shift_head", [(20, 19), (31, 24), (-3, -2), (17, 0)])
def test_shift_outside_0_16_every_tensor(shift_silu, shift_head):
    ir = rescaled(shift_silu, shift_head)
    sess = GraphSession(ir, max_batch=2)
    imgs = random_images(2, 64, seed=40 + shift_silu)
    out = sess.run_yolo_monolithic(imgs)
    for b in range(2):
        ref = O.run_image(ir, imgs[b])
        for name in ref:
            assert np.array_equal(sess.read_tensor(name, batch=2)[b], ref[name]), f"image {b} tensor {name}"
        assert np.array_equal(out["raw_output"][b], O.egress_int8(ir, ref))
    sess.close()
