"""ctypes binding of the reference's own letterbox ingress, pipelines/preprocess_simd.c
fused_preprocess_bgr_to_c8_plane, built from the reference's sources by oracle/build_ref.sh into
oracle/_ref/preprocess_simd.so. Test infrastructure: the checker for the GPU letterbox."""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Optional

import numpy as np

REF_SO = Path(__file__).resolve().parents[2] / "oracle" / "_ref" / "preprocess_simd.so"


def load() -> Optional[C.CDLL]:
    if not REF_SO.exists():
        return None
    lib = C.CDLL(str(REF_SO))
    lib.fused_preprocess_bgr_to_c8_plane.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                                     C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int),
                                                     C.POINTER(C.c_int), C.POINTER(C.c_float)]
    lib.fused_preprocess_bgr_to_c8_plane.restype = C.c_int
    return lib


def letterbox(lib, frame_bgr: np.ndarray, dst_w: int, dst_h: int, lut_q: np.ndarray):
    """uint8 HxWx3 BGR frame -> (uint8 [dst_h][dst_w][3] quantized plane q, (pad_top, pad_left, scale))."""
    f = np.ascontiguousarray(frame_bgr)
    halo = 1
    plane = np.zeros((dst_h + 2 * halo, dst_w + 2 * halo, 8), dtype=np.uint8)
    lut = np.ascontiguousarray(lut_q, dtype=np.uint8)
    top, left, scale = C.c_int(), C.c_int(), C.c_float()
    rc = lib.fused_preprocess_bgr_to_c8_plane(f.ctypes.data, f.shape[1], f.shape[0], f.strides[0], plane.ctypes.data,
                                              dst_w, dst_h, halo, lut.ctypes.data, C.byref(top), C.byref(left),
                                              C.byref(scale))
    if rc != 0:
        raise RuntimeError(f"reference letterbox failed ({rc})")
    return plane[halo:halo + dst_h, halo:halo + dst_w, :3].copy(), (top.value, left.value, scale.value)
