"""GPU decode + NMS against the reference's own decode, bit for bit: the golden detections
(tests/golden/decode_golden.npz, made by the reference's decode_native.c) and, where
oracle/_ref holds the reference decode, live comparisons on the engine's 640x640 heads."""
import numpy as np
import pytest

from ignite_xdna_b200 import InferenceSession, build_yolov8, random_images
from ignite_xdna_b200 import decode as D
from ignite_xdna_b200.heads import layout_from_plan
from ignite_xdna_b200.plan import build_plan

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_gpu_decode_matches_golden(golden_dir):
    import torch
    g = dict(np.load(golden_dir / "decode_golden.npz"))
    layout = layout_from_plan(build_plan(build_yolov8("n", imgsz=160), 4))
    heads = torch.from_numpy(g["heads"]).cuda()
    B = heads.shape[0]
    for ci, (conf, iou, pt, pl, sc) in enumerate(g["cases"]):
        dec = D.GpuDecoder(layout, 160, torch.device("cuda"), conf=float(conf), iou=float(iou))
        lb = np.tile(np.array([pt, pl, sc], dtype=np.float32), (B, 1))
        det = dec(heads, B, letterbox=lb)
        for i in range(B):
            assert np.array_equal(_bits(det[i].boxes), _bits(g[f"c{ci}_i{i}_boxes"])), (ci, i)
            assert np.array_equal(_bits(det[i].scores), _bits(g[f"c{ci}_i{i}_scores"])), (ci, i)
            assert np.array_equal(det[i].classes, g[f"c{ci}_i{i}_classes"]), (ci, i)


@pytest.mark.parametrize("conf,iou", [(0.25, 0.5), (0.05, 0.6)])
def test_gpu_decode_matches_reference_at_640(conf, iou):
    import ref_decode
    lib = ref_decode.load()
    if lib is None:
        pytest.skip("oracle/_ref/decode_native.so is not built")
    import torch
    sess = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=3)
    imgs = random_images(3, 640, seed=12)
    raw = np.array(sess.run(imgs))
    dec = D.GpuDecoder(sess.layout, 640, torch.device("cuda"), conf=conf, iou=iou)
    egress = sess.arena[sess.plan.egress_offset:sess.plan.egress_offset + 3 * sess.out_bytes]
    lb = np.array([[0, 0, 1], [80, 0, 0.5], [3, 5, 1.5]], dtype=np.float32)
    det = dec(egress, 3, letterbox=lb)
    anchors = D.anchor_grid(640)
    tables = []
    for bname, cname in D.HEAD_PAIRS:
        bs, cs = sess.layout.spec(bname), sess.layout.spec(cname)
        sig = D.sigmoid_table(cs.scale, 0)
        tables.append((D.dfl_exp_table(bs.scale, 0), sig, D.sigmoid_low_table(sig), D.q_threshold(conf, cs.scale, 0)))
    for i in range(3):
        b, s, c = ref_decode.decode(lib, raw[i], sess.layout, tables, anchors, conf, iou, tuple(lb[i]))
        assert len(s) == len(det[i].scores)
        assert np.array_equal(_bits(det[i].boxes), _bits(b)) and np.array_equal(_bits(det[i].scores), _bits(s))
        assert np.array_equal(det[i].classes, c)
    sess.close()


def test_gpu_decode_class_pick_with_saturated_sigmoid():
    """Class heads read at scale 0.5: the float32 sigmoid is 1.0 from q = 34 up, so many anchors
    have an earlier class whose byte is below the maximum but shares its score. The numpy argmax
    of the reference picks that earlier class; the kernel's walk through the class bytes must
    too (the maximum's first class alone would differ)."""
    import dataclasses
    import ref_decode
    lib = ref_decode.load()
    if lib is None:
        pytest.skip("oracle/_ref/decode_native.so is not built")
    import torch
    sess = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=2)
    imgs = random_images(2, 640, seed=21)
    raw = np.array(sess.run(imgs))
    cls_names = {c for _, c in D.HEAD_PAIRS}
    layout = dataclasses.replace(sess.layout, heads=tuple(
        dataclasses.replace(h, scale=0.5) if h.name in cls_names else h for h in sess.layout.heads))
    conf, iou = 0.9, 0.6
    # the case this test exists for occurs: an anchor whose first class reaching the saturated
    # score comes before the first class holding the maximum byte
    views = layout.unpack(raw)
    sig = D.sigmoid_table(0.5, 0)
    low = D.sigmoid_low_table(sig)
    ties = 0
    for _, cname in D.HEAD_PAIRS:
        q = views[cname][0].reshape(views[cname].shape[1], -1).astype(np.int32)
        qmax = q.max(axis=0)
        lo = low[qmax + 128]
        ties += int(np.sum((q >= lo).argmax(axis=0) != q.argmax(axis=0)))
    assert ties > 0
    dec = D.GpuDecoder(layout, 640, torch.device("cuda"), conf=conf, iou=iou)
    egress = sess.arena[sess.plan.egress_offset:sess.plan.egress_offset + 2 * sess.out_bytes]
    lb = np.array([[0, 0, 1], [0, 0, 1]], dtype=np.float32)
    det = dec(egress, 2, letterbox=lb)
    anchors = D.anchor_grid(640)
    tables = []
    for bname, cname in D.HEAD_PAIRS:
        bs, cs = layout.spec(bname), layout.spec(cname)
        s = D.sigmoid_table(cs.scale, 0)
        tables.append((D.dfl_exp_table(bs.scale, 0), s, D.sigmoid_low_table(s), D.q_threshold(conf, cs.scale, 0)))
    for i in range(2):
        b, s, c = ref_decode.decode(lib, raw[i], layout, tables, anchors, conf, iou, tuple(lb[i]))
        assert len(s) == len(det[i].scores) and len(s) > 0
        assert np.array_equal(_bits(det[i].boxes), _bits(b)) and np.array_equal(_bits(det[i].scores), _bits(s))
        assert np.array_equal(det[i].classes, c)
    sess.close()
