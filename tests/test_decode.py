"""Host side of the GPU decode: the restated tables against the reference's (golden hashes), and
the reference's own decode (oracle/_ref, when built here) against the golden detections."""
import hashlib
import json

import numpy as np
import pytest

from ignite_xdna_b200 import build_yolov8
from ignite_xdna_b200 import decode as D
from ignite_xdna_b200.heads import HEAD_NAMES, layout_from_plan
from ignite_xdna_b200.plan import build_plan


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest() if a is not None else "none"


@pytest.fixture(scope="module")
def golden(golden_dir):
    return dict(np.load(golden_dir / "decode_golden.npz")), json.loads((golden_dir / "decode_tables.json").read_text())


def layout160():
    return layout_from_plan(build_plan(build_yolov8("n", imgsz=160), 4))


def test_tables_match_the_reference(golden):
    _, meta = golden
    layout = layout160()
    for name in HEAD_NAMES:
        s = layout.spec(name)
        if name.endswith("box"):
            assert sha(D.dfl_exp_table(s.scale, 0)) == meta["tables"][f"{name}_dfl"], name
        else:
            sig = D.sigmoid_table(s.scale, 0)
            assert sha(sig) == meta["tables"][f"{name}_sigmoid"], name
            assert sha(D.sigmoid_low_table(sig)) == meta["tables"][f"{name}_low"], name


def test_anchor_grid():
    ax, ay, st = D.anchor_grid(640)
    assert ax.size == 8400 and ax[0] == 0.5 and ay[80] == 1.5 and st[6399] == 8 and st[6400] == 16 and st[-1] == 32
    assert ax[6400] == 0.5 and ax[8399] == 19.5 and ay[8399] == 19.5


def test_reference_decode_reproduces_golden(golden):
    import ref_decode
    lib = ref_decode.load()
    if lib is None:
        pytest.skip("oracle/_ref/decode_native.so is not built (oracle/build_ref.sh)")
    g, _ = golden
    layout = layout160()
    anchors = (g["anchors_x"], g["anchors_y"], g["strides"])
    for ci, (conf, iou, pt, pl, sc) in enumerate(g["cases"]):
        tables = []
        for bname, cname in D.HEAD_PAIRS:
            bs, cs = layout.spec(bname), layout.spec(cname)
            sig = D.sigmoid_table(cs.scale, 0)
            tables.append((D.dfl_exp_table(bs.scale, 0), sig, D.sigmoid_low_table(sig), D.q_threshold(conf, cs.scale, 0)))
        for i in range(g["heads"].shape[0]):
            b, s, c = ref_decode.decode(lib, g["heads"][i], layout, tables, anchors, conf, iou, (pt, pl, sc))
            assert np.array_equal(b.view(np.uint32), g[f"c{ci}_i{i}_boxes"].view(np.uint32))
            assert np.array_equal(s.view(np.uint32), g[f"c{ci}_i{i}_scores"].view(np.uint32))
            assert np.array_equal(c, g[f"c{ci}_i{i}_classes"])


def test_dense_decode_restatement_equals_the_reference(golden_dir):
    """InferenceSession.decode_yolo_predictions (numpy) against the reference's own
    runtime/session.py decode_yolo_predictions on the same int8 heads (tests/golden/make_dense_golden.py)."""
    from ignite_xdna_b200.session import InferenceSession
    g = np.load(golden_dir / "dense_golden.npz")
    names = [str(n) for n in g["names"]]
    heads = {}
    for n, off, shp in zip(names, g["offsets"], g["shapes"]):
        size = int(np.prod(shp))
        heads[n] = g["egress"][:, off:off + size].reshape((2,) + tuple(int(x) for x in shp))
    heads["scales"] = {n: (float(s), 0) for n, s in zip(names, g["scales"])}
    out = InferenceSession.decode_yolo_predictions(heads)
    np.testing.assert_array_equal(out, g["out"])
