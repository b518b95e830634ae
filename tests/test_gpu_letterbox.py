"""GPU letterbox ingress against the reference's own fused_preprocess_bgr_to_c8_plane: the golden
hashes (tests/golden/letterbox_golden.json, made by the reference's C) over frame sizes that crop,
pad, upscale and keep the image; and a letterboxed run that equals the oracle on the same plane."""
import hashlib
import json

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import InferenceSession

pytestmark = pytest.mark.gpu


def frame(w, h, seed):
    return np.random.default_rng(seed).integers(0, 256, size=(h, w, 3), dtype=np.uint8)


@pytest.fixture(scope="module")
def sess():
    s = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=2)
    yield s
    s.close()


def read_plane(sess, b=0):
    st = sess.plan.input_store
    n = (st.height + 2) * (st.width + 4) * 8
    raw = sess.arena[st.offset + b * n:st.offset + (b + 1) * n].cpu().numpy().view(np.int8)
    v = raw.reshape(st.height + 2, st.width + 4, 8)[1:st.height + 1, 1:st.width + 1, :3]
    return (v.astype(np.int16) + 128).astype(np.uint8)


def test_letterbox_matches_reference_golden(sess, golden_dir):
    for case in json.loads((golden_dir / "letterbox_golden.json").read_text()):
        (top, left), scale = sess.stage_image(frame(case["w"], case["h"], case["seed"]))
        assert (top, left) == (case["pad_top"], case["pad_left"]) and np.float32(scale) == np.float32(case["scale"])
        assert hashlib.sha256(read_plane(sess).tobytes()).hexdigest() == case["sha256"], case


def test_letterboxed_batch_runs_like_the_oracle(sess):
    frames = np.stack([frame(1280, 720, 11), frame(1280, 720, 12)])
    lb = sess.stage_images(frames)
    assert lb.shape == (2, 3) and lb[0, 0] == 140 and lb[0, 2] == 0.5
    planes = [read_plane(sess, b) for b in range(2)]
    out = sess.run_yolo_monolithic(None)
    for b in range(2):
        # the oracle on the same quantized plane (q domain -> its own input tensor)
        ref = O.run_direct(sess.ir, planes[b].transpose(2, 0, 1))
        assert np.array_equal(out["raw_output"][b], O.egress_int8(sess.ir, ref))
