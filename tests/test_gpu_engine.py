"""Whole-network parity on a B200 through the C ABI: every int8 activation and head tensor
must equal the oracle (and, at 640x640, the reference's own run_direct hashes) byte for byte."""
import hashlib
import json

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import InferenceSession, build_yolov8, random_images
from ignite_xdna_b200 import _lib as L

pytestmark = pytest.mark.gpu


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def hashes(golden_dir):
    return json.loads((golden_dir / "graph_hashes.json").read_text())


@pytest.mark.parametrize("imgsz,batch,sms", [(64, 2, None), (96, 3, None), (128, 1, None), (64, 2, "1"),
                                            (96, 3, "2"), (128, 2, "4")])
def test_small_graph_every_tensor(imgsz, batch, sms, monkeypatch):
    """sms forces the launch planner's SM count, so small inputs also run 256/512-row tiles."""
    if sms:
        monkeypatch.setenv("IXB_SM_COUNT", sms)
    sess = InferenceSession.from_spec("yolov8n", imgsz=imgsz, max_batch=batch)
    imgs = random_images(batch, imgsz, seed=21 + imgsz)
    out = sess.run_yolo_monolithic(imgs)
    for b in range(batch):
        ref = O.run_image(sess.ir, imgs[b])
        for name in ref:
            got = sess.read_tensor(name, batch=batch)[b]
            assert np.array_equal(got, ref[name]), f"image {b} tensor {name}"
        assert np.array_equal(out["raw_output"][b], O.egress_int8(sess.ir, ref))
    sess.close()


@pytest.mark.parametrize("imgsz,batch", [(64, 2), (96, 3)])
def test_im2col_stride2_every_tensor(imgsz, batch, monkeypatch):
    """IXB_S2D=0: the stride-2 3x3 convs load their A operand with TMA im2col (IM2COL mode) instead
    of bulk copies of their input's space-to-depth view; every tensor must still equal the oracle."""
    monkeypatch.setenv("IXB_S2D", "0")
    sess = InferenceSession.from_spec("yolov8n", imgsz=imgsz, max_batch=batch)
    assert sum(c.mode == L.MODE_IM2COL for c in sess.plan.convs) == 6
    imgs = random_images(batch, imgsz, seed=7 + imgsz)
    out = sess.run_yolo_monolithic(imgs)
    for b in range(batch):
        ref = O.run_image(sess.ir, imgs[b])
        for name in ref:
            assert np.array_equal(sess.read_tensor(name, batch=batch)[b], ref[name]), f"image {b} tensor {name}"
        assert np.array_equal(out["raw_output"][b], O.egress_int8(sess.ir, ref))
    sess.close()


@pytest.mark.parametrize("imgsz,batch", [(64, 2), (96, 3)])
def test_gathered_upsample_every_tensor(imgsz, batch, monkeypatch):
    """IXB_UP2=0: the concat convs read the upsampled tensors through per-row gathers (GATHER mode)
    instead of the producers' 2x2-replicated copies; every tensor must still equal the oracle."""
    monkeypatch.setenv("IXB_UP2", "0")
    sess = InferenceSession.from_spec("yolov8n", imgsz=imgsz, max_batch=batch)
    assert sum(c.mode == L.MODE_GATHER for c in sess.plan.convs) == 2
    imgs = random_images(batch, imgsz, seed=5 + imgsz)
    out = sess.run_yolo_monolithic(imgs)
    for b in range(batch):
        ref = O.run_image(sess.ir, imgs[b])
        for name in ref:
            assert np.array_equal(sess.read_tensor(name, batch=batch)[b], ref[name]), f"image {b} tensor {name}"
        assert np.array_equal(out["raw_output"][b], O.egress_int8(sess.ir, ref))
    sess.close()


@pytest.mark.parametrize("imgsz,batch,sms", [(64, 2, None), (96, 2, "2")])
def test_pose_graph_every_tensor(imgsz, batch, sms, monkeypatch):
    """YOLOv8-pose: one-class heads and 51-channel keypoint convs run on zero-padded 16-channel
    chunks; every stored tensor and all nine heads equal the oracle."""
    if sms:
        monkeypatch.setenv("IXB_SM_COUNT", sms)
    sess = InferenceSession.from_spec("yolov8n-pose", imgsz=imgsz, max_batch=batch)
    assert len(sess.head_names) == 9
    imgs = random_images(batch, imgsz, seed=5 + imgsz)
    out = sess.run_yolo_monolithic(imgs)
    for b in range(batch):
        ref = O.run_image(sess.ir, imgs[b])
        for name in ref:
            got = sess.read_tensor(name, batch=batch)[b]
            assert np.array_equal(got, ref[name]), f"image {b} tensor {name}"
        assert np.array_equal(out["raw_output"][b], O.egress_int8(sess.ir, ref))
        assert out["p3_kpt"][b].shape == (51, imgsz // 8, imgsz // 8)
    sess.close()


def test_pose_640_matches_reference_hashes(golden_dir):
    h = json.loads((golden_dir / "pose_hashes.json").read_text())["yolov8n-pose"]
    sess = InferenceSession.from_spec("yolov8n-pose", imgsz=640, max_batch=1)
    out = sess.run_yolo_monolithic(random_images(1, 640, seed=h["image_seed"]))
    for name, v in h["heads"].items():
        assert sha(out[name][0]) == v, name
    for name, v in h["tensors"].items():
        assert sha(sess.read_tensor(name, batch=1)[0]) == v, name
    sess.close()


@pytest.mark.parametrize("model", ["yolov8n", "yolov8n-pose"])
def test_branch_groups_equal_the_serial_order(model, monkeypatch):
    """Independent convs of a dependency level run concurrently on forked streams; the result
    equals the graph's own serial order, tensor for tensor (the eager, graph-less fork/join is
    covered by test_graph_replay_equals_layer_by_layer_launches)."""
    imgs = random_images(4, 320, seed=77)
    outs = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("IXB_BRANCHES", flag)
        sess = InferenceSession.from_spec(model, imgsz=320, max_batch=4)
        assert any(k & L.OP_WITH_PREV for k, _ in sess.plan.ops) == (flag == "1")
        out = sess.run_yolo_monolithic(imgs)["raw_output"].copy()
        tensors = {n: sess.read_tensor(n, batch=4) for n in list(sess.ir.tensors)[-20:]}
        outs[flag] = (out, tensors)
        sess.close()
    assert np.array_equal(outs["1"][0], outs["0"][0])
    for n in outs["0"][1]:
        assert np.array_equal(outs["1"][1][n], outs["0"][1][n]), n
    ref = O.run_batch_egress(build_yolov8("n", imgsz=320, task="pose" if "pose" in model else "detect"), imgs[:1])
    assert np.array_equal(outs["1"][0][:1], ref)


def test_yolov8n_640_matches_reference_hashes(hashes):
    h = hashes["yolov8n"]
    sess = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=2)
    imgs = np.concatenate([random_images(1, 640, seed=h["image_seed"]), random_images(1, 640, seed=99)])
    out = sess.run_yolo_monolithic(imgs)
    for name, v in h["tensors"].items():
        got = sess.read_tensor(name, batch=2)[0]
        assert sha(got) == v, name
    for name, v in h["heads"].items():
        assert sha(out[name][0]) == v, name
    ref1 = O.run_batch_egress(sess.ir, imgs[1:2])
    assert np.array_equal(out["raw_output"][1:2], ref1)
    sess.close()


@pytest.mark.parametrize("variant", ["s", "m"])
def test_yolov8sm_640_heads_match_reference_hashes(hashes, variant):
    h = hashes[f"yolov8{variant}"]
    sess = InferenceSession.from_spec(f"yolov8{variant}", imgsz=640, max_batch=1)
    out = sess.run_yolo_monolithic(random_images(1, 640, seed=h["image_seed"]))
    for name, v in h["heads"].items():
        assert sha(out[name][0]) == v, name
    for name, v in h["tensors"].items():
        assert sha(sess.read_tensor(name, batch=1)[0]) == v, name
    sess.close()


def test_batch64_rows_are_independent_and_exact():
    """Each image's heads in a batch of 64 equal a separate run of that image, and the oracle."""
    sess = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=64)
    imgs = random_images(64, 640, seed=5)
    full = np.array(sess.run_yolo_monolithic(imgs)["raw_output"])
    for j in (0, 17, 63):
        one = np.array(sess.run_yolo_monolithic(imgs[j:j + 1])["raw_output"])
        assert np.array_equal(full[j], one[0]), j
    part = np.array(sess.run_yolo_monolithic(imgs[20:27])["raw_output"])
    assert np.array_equal(full[20:27], part)
    assert np.array_equal(full[63:64], O.run_batch_egress(sess.ir, imgs[63:64]))
    sess.close()


def test_graph_replay_equals_layer_by_layer_launches():
    import ctypes as C
    sess = InferenceSession.from_spec("yolov8n", imgsz=96, max_batch=4)
    imgs = random_images(4, 96, seed=8)
    a = np.array(sess.run_yolo_monolithic(imgs)["raw_output"])
    sess.stage_input(imgs)
    L.check(sess.lib.ixb_session_run(sess._h, None, 4, None, L.IN_DEVICE | L.OUT_DEVICE | L.NO_GRAPH))
    b = sess.read_heads(batch=4)
    assert np.array_equal(a, b)
    sess.close()


def test_int8_preprocessor_input_equals_uint8_pixels():
    sess = InferenceSession.from_spec("yolov8n", imgsz=64, max_batch=2)
    imgs = random_images(2, 64, seed=4)
    a = np.array(sess.run(imgs))
    b = np.array(sess.run((imgs.astype(np.int16) - 128).astype(np.int8)))
    assert np.array_equal(a, b)
    sess.close()


def test_device_input_and_staged_dispatch_paths():
    import torch
    sess = InferenceSession.from_spec("yolov8n", imgsz=64, max_batch=2)
    imgs = random_images(2, 64, seed=6)
    ref = O.run_batch_egress(sess.ir, imgs)
    dev = torch.from_numpy(imgs).cuda()
    assert np.array_equal(np.array(sess.run(dev)), ref)
    sess.stage_input(imgs)
    sess.dispatch()
    assert np.array_equal(sess.read_heads(batch=2), ref)
    out = sess.run_yolo_monolithic(None)
    assert np.array_equal(out["raw_output"], ref)
    sess.close()


def test_profile_reports_every_op():
    sess = InferenceSession.from_spec("yolov8n", imgsz=128, max_batch=2)
    ms = sess.profile(2, iters=2)
    assert len(ms) == len(sess.plan.ops) and all(v > 0 for v in ms)
    assert sess.launches(2) == 1 + len(sess.plan.ops)
    tr = sess.trace(2, iters=2)
    conv = [t for t in tr if t is not None]
    assert len(conv) == len(sess.plan.convs)
    assert all(0 <= s <= r <= e for s, r, e in conv)
    groups = []   # an op flagged OP_WITH_PREV runs beside the ops before it (a branch group)
    for (kind, _), t in zip(sess.plan.ops, tr):
        if not (kind & L.OP_WITH_PREV) or not groups:
            groups.append([])
        if t is not None:
            groups[-1].append(t)
    last = 0
    for g in filter(None, groups):   # a group starts after the whole group before it has ended
        assert min(e for _, _, e in g) >= last
        last = max(e for _, _, e in g)
    assert last < 10_000                                   # the whole run within 10 ms
    a = sess.run(random_images(2, 128, seed=5))            # the session's own graph is untouched
    assert np.array_equal(a, O.run_batch_egress(sess.ir, random_images(2, 128, seed=5)))
    sess.close()


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_submitted_runs_match_synchronous_runs(depth):
    """Pipelined submits (a ring of ``depth`` slots, three streams) return the same heads as
    ``run``, in order, whether waited at once, several in flight, or retired by a later submit;
    mixed batch sizes."""
    import torch
    sess = InferenceSession.from_spec("yolov8n", imgsz=96, max_batch=4, pipeline_depth=depth)
    batches = [random_images(b, 96, seed=40 + i) for i, b in enumerate((4, 3, 4, 1, 2, 4))]
    ref = [np.array(sess.run(x)) for x in batches]
    hs = [sess.run_async(x) for x in batches[:2]]
    assert np.array_equal(hs[0].wait(), ref[0]) and np.array_equal(hs[1].wait(), ref[1])
    # four submits without waiting: submits beyond the ring's depth retire the oldest runs
    hs = [sess.run_async(torch.from_numpy(x).pin_memory() if i % 2 else x) for i, x in enumerate(batches[2:])]
    for h, r in zip(hs, ref[2:]):
        assert np.array_equal(h.wait(), r)
    assert hs[0].wait() is hs[0].wait()
    # caller-provided output buffer, device input
    out = np.zeros((4, sess.out_bytes), dtype=np.int8)
    h = sess.run_async(torch.from_numpy(batches[0]).cuda(), out=out)
    h.wait()
    assert np.array_equal(out, ref[0])
    # a synchronous run after submits drains them first
    h = sess.run_async(batches[1])
    assert np.array_equal(np.array(sess.run(batches[3])), ref[3])
    assert np.array_equal(h.wait(), ref[1])
    sess.close()


def test_container_opens_and_matches_reference_hashes(hashes, tmp_path):
    """InferenceSession.from_file on an .ignite container (written by the engine's container writer,
    which reproduces the reference's IgniteModelWriter byte for byte): the heads at 640x640 equal the
    reference's own run_direct hashes."""
    from ignite_xdna_b200 import save_graph
    h = hashes["yolov8n"]
    p = tmp_path / "yolov8n.ignite"
    save_graph(build_yolov8("n", imgsz=640), p)
    sess = InferenceSession.from_file(p, max_batch=1)
    out = sess.run_yolo_monolithic(random_images(1, 640, seed=h["image_seed"]))
    for name, v in h["heads"].items():
        assert sha(out[name][0]) == v, name
    sess.close()


@pytest.mark.parametrize("variant", ["s", "m"])
def test_yolov8sm_batch32_rows_are_independent_and_exact(variant):
    """YOLOv8s / YOLOv8m at the batch of their benchmark configuration (32 per GPU, 640x640): rows of
    the batch equal separate runs of those images, and one row equals the oracle."""
    sess = InferenceSession.from_spec(f"yolov8{variant}", imgsz=640, max_batch=32)
    imgs = random_images(32, 640, seed=50)
    full = np.array(sess.run_yolo_monolithic(imgs)["raw_output"])
    for j in (0, 31):
        assert np.array_equal(full[j], np.array(sess.run_yolo_monolithic(imgs[j:j + 1])["raw_output"])[0]), j
    part = np.array(sess.run_yolo_monolithic(imgs[9:14])["raw_output"])
    assert np.array_equal(full[9:14], part)
    assert np.array_equal(full[31:32], O.run_batch_egress(sess.ir, imgs[31:32]))
    sess.close()
