"""The decode kernel's float screen of same-class NMS pairs (csrc/ixb_decode.cuh,
screen_same_class) never contradicts the exact rule it stands in for.

The exact rule is OpenCV's NMSBoxesBatched overlap test as the reference's
pipelines/decode_native.c applies it (class-offset boxes in double, Rect2d intersection,
overlap 1 - (float)(1 - inter / union), suppress when it is above the IoU threshold). The
screen restated here with numpy float32 (one rounding per operation, as the kernel without FMA
contraction; a contracted FMA only rounds less) must, whenever it decides, agree with it:
random boxes over five decades of size, pairs built to sit within ~1e-6 of the threshold, and
pairs one ulp apart, with class offsets up to ~1.6e5.
"""
import numpy as np

f32 = np.float32
DBL_EPS = np.finfo(np.float64).eps


def _inter_area(ax, ay, aw, ah, bx, by, bw, bh):
    if aw <= 0 or ah <= 0 or bw <= 0 or bh <= 0:
        return 0.0
    a_left, a_top = ax < bx, ay < by
    xmin_x, xmin_w, xmax_x, xmax_w = (ax, aw, bx, bw) if a_left else (bx, bw, ax, aw)
    ymin_y, ymin_h, ymax_y, ymax_h = (ay, ah, by, bh) if a_top else (by, bh, ay, ah)
    if (xmin_x < 0 and xmin_x + xmin_w < xmax_x) or (ymin_y < 0 and ymin_y + ymin_h < ymax_y):
        return 0.0
    w = min(xmax_w, xmin_w - (xmax_x - xmin_x))
    h = min(ymax_h, ymin_h - (ymax_y - ymin_y))
    return 0.0 if (w <= 0 or h <= 0) else w * h


def exact_suppresses(bi, bk, iou, off):
    ix, iy, iw, ih = float(bi[0]) + off, float(bi[1]) + off, float(bi[2]), float(bi[3])
    kx, ky, kw, kh = float(bk[0]) + off, float(bk[1]) + off, float(bk[2]), float(bk[3])
    ia, ka = iw * ih, kw * kh
    if ia + ka <= DBL_EPS:
        ov = f32(1.0)
    else:
        inter = _inter_area(ix, iy, iw, ih, kx, ky, kw, kh)
        ov = f32(f32(1.0) - f32(1.0 - inter / (ia + ka - inter)))
    return not (ov <= f32(iou))


def screen(a, b, iou):
    a = [f32(v) for v in a]
    b = [f32(v) for v in b]
    iou = f32(iou)
    ax2, ay2, bx2, by2 = a[0] + a[2], a[1] + a[3], b[0] + b[2], b[1] + b[3]
    iw = min(ax2, bx2) - max(a[0], b[0])
    ih = min(ay2, by2) - max(a[1], b[1])
    inter = iw * ih if (iw > 0 and ih > 0) else f32(0)
    aa, ab = a[2] * a[3], b[2] * b[3]
    uni = (aa + ab) - inter
    m = max(abs(a[0]), abs(ax2), abs(a[1]), abs(ay2), abs(b[0]), abs(bx2), abs(b[1]), abs(by2))
    delta = m * f32(2.0 ** -22)
    per = (a[2] + a[3]) + (b[2] + b[3])
    err = f32(2) * delta * (per + delta) + f32(2.0 ** -21) * (aa + ab + uni + inter)
    margin = err + f32(2e-6) * uni
    d = inter - iou * uni
    if d > margin:
        return 1
    if d < -margin:
        return 0
    return -1


def test_float_screen_agrees_with_exact_rule():
    rng = np.random.default_rng(7)
    decided = 0
    with np.errstate(over="ignore", invalid="ignore"):
        for trial in range(20000):
            kind = trial % 4
            scale = 10 ** rng.uniform(-2, 3.3)
            a = np.array([rng.uniform(-0.3, 1) * scale, rng.uniform(-0.3, 1) * scale,
                          rng.uniform(0, 1) * scale, rng.uniform(0, 1) * scale], np.float32)
            iou = f32(rng.choice([0.45, 0.5, 0.7, 0.3, 0.0, 1.0, rng.uniform(0, 1)]))
            if kind == 0:
                b = np.array([a[0] + rng.normal() * a[2] * 0.3, a[1] + rng.normal() * a[3] * 0.3,
                              a[2] * rng.uniform(0.5, 1.5), a[3] * rng.uniform(0.5, 1.5)], np.float32)
            elif kind == 1:  # b is a shifted along x so that the IoU is within ~1e-6 of the threshold
                s = a[2] * (1 - float(iou)) / (1 + float(iou)) * (1 + rng.normal() * 1e-6)
                b = np.array([a[0] + s, a[1], a[2], a[3]], np.float32)
            elif kind == 2:
                b = np.array([a[0] + rng.uniform(-1, 1) * scale, a[1] + rng.uniform(-1, 1) * scale,
                              rng.uniform(0, 1) * scale, rng.uniform(0, 1) * scale], np.float32)
            else:  # one ulp apart
                b = a.copy()
                b[2] = np.nextafter(b[2], np.float32(np.inf))
                b[0] = np.nextafter(b[0], np.float32(-np.inf))
            off = float(rng.integers(0, 80)) * float(rng.uniform(600, 2000))
            r = screen(a, b, iou)
            if r >= 0:
                decided += 1
                assert bool(r) == exact_suppresses(a, b, iou, off), (a, b, iou, off)
    assert decided > 10000   # the screen decides most pairs
