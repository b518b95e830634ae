"""Failure paths on a B200, made without a GPU fault: host waits that run out, and a device wait
that nothing completes (the kernel gives up after its limit, raises the device flag and returns).
After each, the session or the context goes on to produce oracle-exact heads."""
import ctypes as C

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import InferenceSession, random_images
from ignite_xdna_b200 import _lib as L

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def big():
    sess = InferenceSession.from_spec("yolov8n", imgsz=640, max_batch=64)
    sess.run(random_images(1, 640, seed=2))       # graphs and launch plans built before the waits
    yield sess
    sess.close()


def test_host_wait_times_out_then_drains(big):
    """ixb_session_wait with 0 ms on a 64-image 640x640 run reports IXB_ERR_TIMEOUT (not fatal);
    the next wait completes the run and its heads equal a plain run's."""
    imgs = random_images(64, 640, seed=11)
    big.stage_input(imgs)
    lib = big.lib
    L.check(lib.ixb_session_run(big._h, None, 64, None, L.IN_DEVICE | L.OUT_DEVICE | L.ASYNC))
    assert lib.ixb_session_wait(big._h, 0) == L.IXB_ERR_TIMEOUT
    assert lib.ixb_session_wait(big._h, 60000) == 0
    heads = big.read_heads(batch=64).copy()
    assert np.array_equal(heads[5], big.run(imgs[5:6])[0])


def test_async_runs_stack(big):
    """Asynchronous runs queue behind a pending one on the session's stream; one wait completes
    them all, and the heads are a plain run's (the session's loop the bench times)."""
    imgs = random_images(64, 640, seed=13)
    big.stage_input(imgs)
    lib = big.lib
    for _ in range(3):
        L.check(lib.ixb_session_run(big._h, None, 64, None, L.IN_DEVICE | L.OUT_DEVICE | L.ASYNC))
    assert lib.ixb_session_wait(big._h, 60000) == 0
    heads = big.read_heads(batch=64).copy()
    assert np.array_equal(heads[17], big.run(imgs[17:18])[0])


def test_ticket_wait_times_out_then_drains(big):
    imgs = random_images(64, 640, seed=12)
    h = big.run_async(imgs)
    with pytest.raises(TimeoutError):
        h.wait(0)
    out = h.wait(60000).copy()
    assert np.array_equal(out[63], big.run(imgs[63:64])[0])


def test_device_bounded_wait_gives_up_and_context_stays_usable():
    lib = L.load()
    for limit_us in (1000, 50000):
        assert lib.ixb_check_wait_timeout(limit_us, None) == L.IXB_ERR_DEVICE
        flag = C.c_int(-1)
        L.check(lib.ixb_device_error(C.byref(flag)))
        assert flag.value == 0           # reported once, then clear
    sess = InferenceSession.from_spec("yolov8n", imgsz=64, max_batch=2)
    imgs = random_images(2, 64, seed=13)
    assert np.array_equal(sess.run(imgs), O.run_batch_egress(sess.ir, imgs))
    sess.close()


def test_sessions_on_two_devices_in_one_process():
    """The kernels' shared-memory limits are raised per device: a second GPU's session runs too."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    imgs = random_images(2, 64, seed=14)
    ref = None
    for dev in (0, 1):
        sess = InferenceSession.from_spec("yolov8n", imgsz=64, max_batch=2, device_index=dev)
        out = sess.run(imgs)
        ref = O.run_batch_egress(sess.ir, imgs) if ref is None else ref
        assert np.array_equal(out, ref), f"device {dev}"
        sess.close()
