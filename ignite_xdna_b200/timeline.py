"""Live per-layer device timeline of one graph run: ``python -m ignite_xdna_b200.timeline [model] [batch]``.

Runs the seeded synthetic graph through ``GraphSession.trace`` (the C ABI's ``ixb_session_trace``:
a copy of the run's CUDA graph whose conv launches mark the global timer) and prints, per op in
execution order, when its first CTA started, when its inputs were ready (the wait for the previous
kernel returned), when its last CTA ended, and the gap before it, in microseconds.
"""
from __future__ import annotations

import sys

from .session import InferenceSession
from .yolov8 import random_images


def timeline(model: str = "yolov8n", batch: int = 64, imgsz: int = 640, iters: int = 5):
    sess = InferenceSession.from_spec(model, imgsz=imgsz, max_batch=batch)
    try:
        sess.run(random_images(batch, imgsz, seed=3))
        rows = []
        prev_end = 0.0
        for (kind, idx), t in zip(sess.plan.ops, sess.trace(batch, iters)):
            if t is None:
                rows.append(("pool", None))
                continue
            d = sess.plan.convs[idx].desc
            start, ready, end = t
            rows.append((f"{idx:3d} {sess.plan.convs[idx].layer.name[:30]:30s} mode {d.mode} k{d.k} "
                         f"{d.cin:4d}->{d.cout:4d} {d.out_h:3d}x{d.out_w:<3d}",
                         (start, ready, end, end - ready, ready - prev_end)))
            prev_end = max(prev_end, end)
        return rows, prev_end
    finally:
        sess.close()


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    model = argv[0] if argv else "yolov8n"
    batch = int(argv[1]) if len(argv) > 1 else 64
    rows, span = timeline(model, batch)
    print(f"{'op':70s} {'start':>8s} {'ready':>8s} {'end':>8s} {'run':>7s} {'gap':>6s}")
    for name, t in rows:
        if t is None:
            print(f"{'    SPPF pool (not marked)':70s}")
        else:
            print(f"{name:70s} {t[0]:8.1f} {t[1]:8.1f} {t[2]:8.1f} {t[3]:7.1f} {t[4]:6.1f}")
    print(f"span {span:.1f} us (first conv start to last conv end)")


if __name__ == "__main__":
    main()
