"""ctypes binding of libixb200.so (include/ixb200.h).

The structures mirror the header field for field; ``load()`` checks their sizes against the
library's own ``ixb_abi_sizes`` before anything is called. There is no fallback: without the
compiled library every GPU entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_NAME = "libixb200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

IXB_OK = 0
ERRORS = {-1: "invalid", -2: "cuda", -3: "timeout", -4: "device", -5: "unsupported", -6: "capacity"}
IXB_ERR_INVALID = -1
IXB_ERR_TIMEOUT = -3
IXB_ERR_DEVICE = -4
IXB_ERR_CAPACITY = -6
IXB_ERR_UNSUPPORTED = -5
MAX_SEGS = 4
API_VERSION = 9
MAX_EXTRA_SLOTS = 3
MODE_WINDOW, MODE_GATHER, MODE_STEM, MODE_IM2COL = 0, 1, 2, 3
OUT2_NONE, OUT2_UP2, OUT2_S2D, OUT2_S2D_ONLY = 0, 1, 2, 3
IN_DEVICE, OUT_DEVICE, ASYNC, NO_GRAPH, IN_STORE = 1, 2, 4, 8, 16
OP_CONV, OP_POOL = 0, 1
OP_WITH_PREV = 0x100     # a conv that runs concurrently with the op(s) before it (branch group)
MAX_BRANCHES = 8


class Segment(C.Structure):
    _fields_ = [("offset", C.c_uint64), ("plane_stride", C.c_uint64), ("chunk_offset", C.c_int32),
                ("channels", C.c_int32), ("height", C.c_int32), ("width", C.c_int32), ("up2", C.c_int32),
                ("guard", C.c_int32)]


class ConvDesc(C.Structure):
    _fields_ = [("mode", C.c_int32), ("k", C.c_int32), ("stride", C.c_int32),
                ("in_h", C.c_int32), ("in_w", C.c_int32), ("out_h", C.c_int32), ("out_w", C.c_int32),
                ("cin", C.c_int32), ("cout", C.c_int32), ("n_tile", C.c_int32), ("cp", C.c_int32),
                ("s2d_in", C.c_int32),
                ("nseg", C.c_int32), ("seg", Segment * MAX_SEGS),
                ("w_offset", C.c_uint64), ("w_bytes", C.c_uint64), ("bias_offset", C.c_uint64),
                ("lut_offset", C.c_uint64), ("shift", C.c_int32), ("has_residual", C.c_int32),
                ("residual", Segment), ("res_lsh_main", C.c_int32), ("res_lsh_res", C.c_int32),
                ("res_shift", C.c_int32), ("out_nchw", C.c_int32), ("out", Segment),
                ("egress_offset", C.c_uint64), ("egress_image_bytes", C.c_uint64),
                ("egress_channels", C.c_int32), ("out2_kind", C.c_int32),
                ("reserved3", C.c_int32), ("out2", Segment)]


class PoolDesc(C.Structure):
    _fields_ = [("inp", Segment), ("out", Segment * 3)]


class Op(C.Structure):
    _fields_ = [("kind", C.c_int32), ("index", C.c_int32)]


class Plan(C.Structure):
    _fields_ = [("api_version", C.c_int32), ("max_batch", C.c_int32), ("img_h", C.c_int32), ("img_w", C.c_int32),
                ("n_convs", C.c_int32), ("n_pools", C.c_int32), ("n_ops", C.c_int32),
                ("convs", C.POINTER(ConvDesc)), ("pools", C.POINTER(PoolDesc)), ("ops", C.POINTER(Op)),
                ("images_offset", C.c_uint64), ("input_lut_offset", C.c_uint64), ("input", Segment),
                ("egress_offset", C.c_uint64), ("egress_image_bytes", C.c_uint64), ("arena_bytes", C.c_uint64),
                ("extra_slots", C.c_int32), ("input_s2d", C.c_int32),
                ("extra_images_offset", C.c_uint64 * MAX_EXTRA_SLOTS),
                ("extra_egress_offset", C.c_uint64 * MAX_EXTRA_SLOTS), ("input_s2d_view", Segment)]


class IxbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ixb error {code} ({ERRORS.get(code, '?')}): {msg}")
        self.code = code


_lib = None

_SIGS = {
    "ixb_last_error": (C.c_char_p, []),
    "ixb_version": (C.c_int, []),
    "ixb_abi_sizes": (C.c_int, [C.POINTER(C.c_uint64), C.c_int]),
    "ixb_device_error": (C.c_int, [C.POINTER(C.c_int)]),
    "ixb_check_wait_timeout": (C.c_int, [C.c_int, C.c_void_p]),
    "ixb_session_create": (C.c_int, [C.POINTER(Plan), C.c_int, C.c_void_p, C.c_uint64, C.POINTER(C.c_void_p)]),
    "ixb_session_destroy": (C.c_int, [C.c_void_p]),
    "ixb_session_arena": (C.c_void_p, [C.c_void_p]),
    "ixb_session_stream": (C.c_void_p, [C.c_void_p]),
    "ixb_session_run": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int]),
    "ixb_session_wait": (C.c_int, [C.c_void_p, C.c_int]),
    "ixb_session_submit": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.POINTER(C.c_uint64)]),
    "ixb_session_wait_ticket": (C.c_int, [C.c_void_p, C.c_uint64, C.c_int]),
    "ixb_session_streams": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                      C.POINTER(C.c_void_p)]),
    "ixb_session_last_ms": (C.c_int, [C.c_void_p, C.POINTER(C.c_float)]),
    "ixb_session_launches": (C.c_int, [C.c_void_p, C.c_int]),
    "ixb_session_profile": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_float)]),
    "ixb_session_trace": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_uint64)]),
    "ixb_conv_layer": (C.c_int, [C.POINTER(ConvDesc), C.c_void_p, C.c_uint64, C.c_int, C.c_void_p]),
    "ixb_conv_layer_stats": (C.c_int, [C.POINTER(ConvDesc), C.c_void_p, C.c_uint64, C.c_int, C.c_void_p,
                                       C.c_void_p, C.c_int64]),
    "ixb_conv_schedule": (C.c_int, [C.POINTER(ConvDesc), C.POINTER(C.c_int32), C.c_int, C.POINTER(C.c_int32),
                                    C.c_int]),
    "ixb_conv_launch_info": (C.c_int, [C.POINTER(ConvDesc), C.c_uint64, C.c_int, C.POINTER(C.c_int32), C.c_int]),
    "ixb_pool_layer": (C.c_int, [C.POINTER(PoolDesc), C.c_void_p, C.c_uint64, C.c_int, C.c_void_p]),
    "ixb_quantize_images": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "ixb_i8gemm_srs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_void_p]),
    "ixb_i8gemm_i32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "ixb_gemm_plan_info": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int32), C.c_int]),
    "ixb_w4a8_image_bytes": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_uint64)]),
    "ixb_w4a8_prepare": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "ixb_w4a8_gemm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                C.c_void_p]),
    "ixb_w4a8_gemv": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "ixb_u8i4_gemm_i32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "ixb_decode_yolo": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_uint64, C.c_void_p, C.c_int32, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "ixb_decode_yolo_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_uint64, C.c_void_p, C.c_int32,
                                          C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "ixb_letterbox_frames": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_void_p,
                                       C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint64, C.POINTER(C.c_float),
                                       C.c_void_p]),
    "ixb_session_letterbox": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                        C.POINTER(C.c_float)]),
    "ixb_decode_dense": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int, C.c_uint64, C.c_void_p, C.c_void_p]),
    "ixb_session_set_detect": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ixb_session_set_thresholds": (C.c_int, [C.c_void_p, C.c_float, C.c_float]),
    "ixb_session_set_class_names": (C.c_int, [C.c_void_p, C.POINTER(C.c_char_p), C.c_int]),
    "ixb_session_submit_detect": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.POINTER(C.c_uint64)]),
    "ixb_session_submit_frames": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint64,
                                            C.POINTER(C.c_uint64)]),
    "ixb_session_detections": (C.c_int, [C.c_void_p, C.c_uint64, C.c_int, C.POINTER(C.c_int32),
                                         C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                         C.POINTER(C.c_void_p)]),
    "ixb_session_wait_detections": (C.c_int, [C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_void_p, C.c_int]),
    "ixb_run_frame": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int]),
    "ixb_session_last_timings": (C.c_int, [C.c_void_p, C.c_void_p]),
}


class DenseHead(C.Structure):
    _fields_ = [("box_offset", C.c_uint64), ("cls_offset", C.c_uint64), ("box_scale", C.c_float),
                ("box_zero_point", C.c_int32), ("cls_scale", C.c_float), ("cls_zero_point", C.c_int32),
                ("grid", C.c_int32), ("stride", C.c_float)]


class Detection(C.Structure):
    _fields_ = [("x0", C.c_float), ("y0", C.c_float), ("w", C.c_float), ("h", C.c_float), ("score", C.c_float),
                ("class_id", C.c_int32), ("class_name", C.c_char * 32)]


class Timings(C.Structure):
    _fields_ = [("preprocess_ms", C.c_double), ("gpu_exec_ms", C.c_double), ("postprocess_ms", C.c_double),
                ("glass_to_glass_ms", C.c_double)]


def exported_symbols():
    return sorted(_SIGS)


def load():
    """The loaded library; raises if it was not built (``python -c 'import __graft_entry__; __graft_entry__.build()'``)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("IXB_LIB", LIB_PATH))
    if not path.exists():
        raise ImportError(f"{path} is missing: build the CUDA extension first (ignite_xdna_b200.build)")
    lib = C.CDLL(str(path))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    sizes = (C.c_uint64 * 4)()
    lib.ixb_abi_sizes(sizes, 4)
    want = [C.sizeof(Segment), C.sizeof(ConvDesc), C.sizeof(PoolDesc), C.sizeof(Plan)]
    if list(sizes) != want:
        raise ImportError(f"ABI mismatch between {path} and this binding: {list(sizes)} vs {want}")
    if lib.ixb_version() != API_VERSION:
        raise ImportError("libixb200 API version mismatch")
    _lib = lib
    return lib


LAUNCH_FIELDS = ("mt", "tile_rows", "m_tiles", "stages", "b_resident", "grid_x", "grid_y", "smem", "tmem_cols",
                 "kblocks", "rows_a", "cp")


def conv_launch_info(desc, arena_bytes: int, batch: int) -> dict:
    info = (C.c_int32 * len(LAUNCH_FIELDS))()
    check(load().ixb_conv_launch_info(C.byref(desc), arena_bytes, batch, info, len(LAUNCH_FIELDS)))
    return dict(zip(LAUNCH_FIELDS, list(info)))


def conv_schedule(desc):
    """The kernel's K schedule of a conv: per K-block {chunk0, nchunks, tap0, ntaps, ops, b_off, b_bytes},
    A slot s holding chunk chunk0 + s // ntaps at tap tap0 + s % ntaps; per MMA ((slot, chunk, tap),
    (slot, chunk, tap) or None) for its two 32-byte K-halves (None: zero weights)."""
    kb = (C.c_int32 * (8 * 512))()
    ops = (C.c_int32 * (6 * 4096))()
    n = check(load().ixb_conv_schedule(C.byref(desc), kb, 512, ops, 4096))
    blocks = []
    for i in range(n):
        c0, nc, t0, nt, op0, nops, boff, bbytes = kb[8 * i:8 * i + 8]
        mm = []
        for j in range(op0, op0 + nops):
            s0, ch0, tp0, s1, ch1, tp1 = ops[6 * j:6 * j + 6]
            mm.append(((s0, ch0, tp0), (s1, ch1, tp1) if ch1 >= 0 else None))
        blocks.append({"chunk0": c0, "nchunks": nc, "tap0": t0, "ntaps": nt, "ops": mm, "b_off": boff,
                       "b_bytes": bbytes})
    return blocks


def check(rc: int) -> int:
    if rc < 0:
        raise IxbError(rc, load().ixb_last_error().decode(errors="replace"))
    return rc
