"""The oracle's signed-domain conv rule (used for negative SRS shifts, which the reference's folded
bias cannot express) equals the reference's folded uint8 rule for every shift it can express."""
import copy

import numpy as np

import ixb_oracle as O
from ignite_xdna_b200 import build_yolov8, random_images


def test_signed_domain_rule_equals_folded_rule_for_nonnegative_shifts():
    ir = build_yolov8("n", imgsz=64)
    L = copy.deepcopy(next(c for c in ir.conv_layers() if c.name.startswith("/model.4/m.0/cv1")))
    x = O.run_image(ir, random_images(1, 64, seed=9)[0])
    src = ir.tensors[L.inputs[0].tensor]
    inp = O.gather_input(x, L.inputs, src.height, src.width)
    for s in (0, 1, 5, 9, 16, 17, 23, 31):
        L.conv_scale *= 2.0 ** (s - L.shift_out)
        folded = O.sat_u8(O.rne_shift(O.conv_accumulate(L, inp), s))
        signed = O.sat_u8(O.rne_shift(O.conv_accumulate(L, inp, folded=False), s) + O.ZP)
        assert np.array_equal(folded, signed), s


def test_negative_shift_is_a_saturating_left_shift():
    ir = build_yolov8("n", imgsz=64)
    L = copy.deepcopy(next(c for c in ir.conv_layers() if c.name.startswith("/model.4/m.0/cv1")))
    L.sigmoid = None
    x = O.run_image(ir, random_images(1, 64, seed=9)[0])
    src = ir.tensors[L.inputs[0].tensor]
    inp = O.gather_input(x, L.inputs, src.height, src.width)
    acc = O.conv_accumulate(L, inp, folded=False)
    L.conv_scale *= 2.0 ** (-2 - L.shift_out)
    got = O.conv_direct(L, inp).astype(np.int64)
    assert np.array_equal(got, np.clip(acc * 4 + 128, 0, 255))
