"""ixb_decode_yolo_noalloc, the decode entry point for callers that may not allocate device memory
(a plugin inside a host application that owns the CUDA context and its memory pool, or a loop that
cannot take cudaMalloc's implicit synchronisation): its scratch is a fixed array inside the library.
Through the C ABI it must give the same detections, bit for bit, as ixb_decode_yolo on the same
heads, on two calls in a row whose tables differ, so that nothing of the first call's scratch
reaches the second. This file is collected last, so a run that stops at its first failure has run
every other test before this one."""
import ctypes as C
import dataclasses

import numpy as np
import pytest

from ignite_xdna_b200 import _lib as L
from ignite_xdna_b200 import build_yolov8
from ignite_xdna_b200 import decode as D
from ignite_xdna_b200.heads import layout_from_plan
from ignite_xdna_b200.plan import build_plan

pytestmark = pytest.mark.gpu


def _decode(lib, fn, dec, heads, batch, lb, cap):
    import torch
    dev = heads.device
    boxes = torch.full((batch, cap, 4), -1.0, dtype=torch.float32, device=dev)
    scores = torch.full((batch, cap), -1.0, dtype=torch.float32, device=dev)
    classes = torch.full((batch, cap), -1, dtype=torch.int32, device=dev)
    counts = torch.full((batch,), -7, dtype=torch.int32, device=dev)
    L.check(getattr(lib, fn)(C.byref(dec.desc), C.c_void_p(heads.data_ptr()), batch, dec.layout.image_bytes,
                             C.c_void_p(lb.data_ptr()), cap, C.c_void_p(boxes.data_ptr()),
                             C.c_void_p(scores.data_ptr()), C.c_void_p(classes.data_ptr()),
                             C.c_void_p(counts.data_ptr()), None))
    torch.cuda.synchronize()
    n = counts.cpu().numpy()
    b, s, c = boxes.cpu().numpy(), scores.cpu().numpy(), classes.cpu().numpy()
    return [(b[i, :n[i]], s[i, :n[i]], c[i, :n[i]]) for i in range(batch)], n


def test_noalloc_decode_equals_decode_on_two_calls():
    import torch
    lib = L.load()
    layout = layout_from_plan(build_plan(build_yolov8("n", imgsz=640), 3))
    cls_names = {c for _, c in D.HEAD_PAIRS}
    # two table sets: the graph's class scales, then 0.5 (a saturating sigmoid: other score ranks)
    layouts = [layout, dataclasses.replace(layout, heads=tuple(
        dataclasses.replace(h, scale=0.5) if h.name in cls_names else h for h in layout.heads))]
    g = torch.Generator(device="cuda").manual_seed(5)
    batch, cap = 3, 8400
    lb = torch.tensor([[0, 0, 1], [80, 0, 0.5], [3, 5, 1.5]], dtype=torch.float32, device="cuda")
    for k, (lay, conf, iou) in enumerate(zip(layouts, (0.25, 0.9), (0.5, 0.6))):
        heads = torch.randint(-128, 128, (batch * lay.image_bytes,), dtype=torch.int8, device="cuda", generator=g)
        dec = D.GpuDecoder(lay, 640, torch.device("cuda"), conf=conf, iou=iou)
        want, n_want = _decode(lib, "ixb_decode_yolo", dec, heads, batch, lb, cap)
        got, n_got = _decode(lib, "ixb_decode_yolo_noalloc", dec, heads, batch, lb, cap)
        assert np.array_equal(n_got, n_want) and (n_want > 0).all(), (k, n_got, n_want)
        for i in range(batch):
            for a, b in zip(got[i], want[i]):
                assert np.array_equal(np.ascontiguousarray(a).view(np.uint32),
                                      np.ascontiguousarray(b).view(np.uint32)), (k, i)
