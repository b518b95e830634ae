"""The detection stage on a B200 through the C ABI: frames or images in, detections out.

* the dense decode kernel (ixb_decode_dense) against the reference's own decode_yolo_predictions
  on fixture heads, and against the numpy restatement on live 640x640 heads (float32 tolerance);
* ticketed detection runs (ixb_session_submit_detect / _submit_frames / _detections) and the
  synchronous ixb_run_frame against the standalone decode kernel on the same heads, bit for bit
  (the decode kernel itself is pinned to the reference's compiled decode_native.c by
  tests/test_gpu_decode.py).
"""
import ctypes as C

import numpy as np
import pytest

from ignite_xdna_b200 import InferenceSession, random_images
from ignite_xdna_b200 import _lib as L
from ignite_xdna_b200.decode import GpuDecoder

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-5, 1e-4     # float32 expf (CUDA) against numpy's float32 exp


def test_dense_kernel_matches_the_reference_decode(golden_dir):
    import torch
    g = np.load(golden_dir / "dense_golden.npz")
    heads = (L.DenseHead * 3)()
    names = [str(n) for n in g["names"]]
    spec = {n: (int(o), tuple(int(x) for x in s), float(sc)) for n, o, s, sc in
            zip(names, g["offsets"], g["shapes"], g["scales"])}
    for h, (lvl, stride) in enumerate(zip((3, 4, 5), (8, 16, 32))):
        bo, bs, bsc = spec[f"p{lvl}_box"]
        co, cs, csc = spec[f"p{lvl}_cls"]
        d = heads[h]
        d.box_offset, d.cls_offset, d.box_scale, d.box_zero_point = bo, co, bsc, 0
        d.cls_scale, d.cls_zero_point, d.grid, d.stride = csc, 0, bs[1], float(stride)
    eg = torch.from_numpy(g["egress"]).cuda()
    out = torch.empty(g["out"].shape, dtype=torch.float32, device="cuda")
    lib = L.load()
    L.check(lib.ixb_decode_dense(heads, 80, C.c_void_p(eg.data_ptr()), 2, eg.shape[1], C.c_void_p(out.data_ptr()),
                                 None))
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], rtol=RTOL, atol=ATOL)


@pytest.fixture(scope="module")
def sess():
    s = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=8)
    yield s
    s.close()


def test_dense_decode_of_live_heads(sess):
    imgs = random_images(3, 640, seed=31)
    out = sess.run_yolo_monolithic(imgs)
    ref = sess.decode_yolo_predictions(out)
    got = sess.decode_predictions(batch=3).cpu().numpy()
    assert got.shape == (3, 84, 8400)
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)


def _decoded_heads(sess, imgs, conf=0.25, iou=0.5, letterbox=None):
    """Reference path: a plain run, then the standalone decode kernel on the device egress."""
    import torch
    b = imgs.shape[0]
    sess.run_yolo_monolithic(imgs)
    dec = GpuDecoder(sess.layout, 640, sess.device, conf=conf, iou=iou)
    eg = sess.arena[sess.plan.egress_offset:sess.plan.egress_offset + b * sess.out_bytes]
    return dec(eg, b, letterbox=letterbox)


def _same(a, b):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert np.array_equal(x.boxes, y.boxes) and np.array_equal(x.scores, y.scores)
        assert np.array_equal(x.classes, y.classes)


def test_submit_detect_equals_the_decode_of_the_heads(sess):
    sess.set_detect(capacity=8400)
    imgs = random_images(8, 640, seed=32)
    lb = np.array([[0.0, 0.0, 1.0], [12.0, 0.0, 0.5], [0.0, 80.0, 0.75]] + [[0.0, 0.0, 1.0]] * 5, np.float32)
    hs = [sess.run_async(imgs, detect=True, letterbox=lb) for _ in range(4)]   # the ring wraps around
    got = [h.wait(60000) for h in hs]
    ref = _decoded_heads(sess, imgs, letterbox=lb)
    for g in got:
        _same(g, ref)
    assert sum(len(d.scores) for d in ref) > 0
    t = sess.last_timings
    assert t["gpu_exec_ms"] > 0 and t["postprocess_ms"] > 0 and t["glass_to_glass_ms"] >= t["gpu_exec_ms"]


def test_thresholds_change_the_detection_stage(sess):
    sess.set_detect(capacity=8400)
    sess.set_thresholds(0.5, 0.45)
    imgs = random_images(2, 640, seed=33)
    got = sess.run_async(imgs, detect=True).wait(60000)
    _same(got, _decoded_heads(sess, imgs, conf=0.5, iou=0.45))


def test_frames_path_equals_letterbox_then_decode(sess):
    """BGR frames of another size: copied in, letterboxed on the GPU, network, decode; the same
    detections as stage_images + run + the standalone decode with the letterbox rows."""
    sess.set_detect(capacity=8400, class_names=[f"c{i}" for i in range(80)])
    rng = np.random.default_rng(34)
    frames = rng.integers(0, 256, size=(3, 360, 500, 3), dtype=np.uint8)
    got = sess.submit_frames(frames).wait(60000)
    lb = sess.stage_images(frames)
    sess.dispatch()
    dec = GpuDecoder(sess.layout, 640, sess.device)
    eg = sess.arena[sess.plan.egress_offset:sess.plan.egress_offset + 3 * sess.out_bytes]
    _same(got, dec(eg, 3, letterbox=lb))
    one = sess.run_frame(frames[1], max_detections=8400)
    assert len(one) == len(got[1].scores)
    for (x0, y0, w, h, sc, c, name), bx, s, k in zip(one, got[1].boxes, got[1].scores, got[1].classes):
        assert (x0, y0, w, h) == tuple(bx) and sc == s and c == k and name == f"c{k}"
    assert sess.last_timings["preprocess_ms"] > 0


def test_capacity_overflow_is_reported(sess):
    sess.set_detect(capacity=1, conf=0.01)
    imgs = random_images(1, 640, seed=35)
    h = sess.run_async(imgs, detect=True)
    with pytest.raises(RuntimeError, match="survive NMS"):
        h.wait(60000)
    sess.set_detect(capacity=8400)
