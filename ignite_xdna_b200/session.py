"""Inference sessions: the reference's runtime surface over the B200 engine.

``GraphSession`` keeps the method names, arguments and return dictionaries of the
reference's ``src/ignite_xdna/runtime/graph_session.py`` ``GraphSession`` (``stage_input``
:891-901, ``dispatch`` :628-651, ``read_heads`` :903-930, ``run_yolo_monolithic`` :932-989,
``run`` :991-992, ``head_status`` :855, ``close``/context manager :764-770, :995) and
``InferenceSession.decode_yolo_predictions`` (``runtime/session.py`` :1223-1278), with a
leading batch dimension: the reference runs one image per dispatch, this engine a batch per
CUDA-graph launch.

PyTorch provides device memory (the arena) and pinned host buffers only; every kernel is
launched by libixb200.so on the session's own stream. There is no CPU path: without the
library or a GPU the session refuses to open.
"""
from __future__ import annotations

import ctypes as C
import time
import warnings
from pathlib import Path
from typing import Any, Dict, Optional, Union

import numpy as np

from . import _lib as L
from .graph import GraphIR
from .heads import HeadStatus, layout_from_plan
from .plan import DevicePlan, build_plan, c_plan


def _torch():
    import torch
    return torch


class RunHandle:
    """One submitted batch in flight (the reference's ``runtime/session.py`` ``RunHandle`` :40-85).

    ``wait`` blocks until the batch's heads are in host memory and returns them as int8
    [B, egress_image_bytes]. Without an ``out`` buffer the result lives in the session's pinned
    egress slot, which the submit ``pipeline_depth`` tickets later reuses: a handle still unwaited
    at that point is completed first and keeps a private copy."""

    def __init__(self, session: "GraphSession", ticket: int, batch: int, egress: np.ndarray, keep: Any):
        self._s = session
        self.ticket = int(ticket)
        self.batch = int(batch)
        self._egress = egress
        self._keep = keep          # host/device input buffers that must outlive the copies
        self._result: Optional[np.ndarray] = None

    @property
    def done(self) -> bool:
        return self._result is not None

    def wait(self, timeout_ms: int = 2000) -> np.ndarray:
        if self._result is None:
            rc = self._s.lib.ixb_session_wait_ticket(self._s._h, C.c_uint64(self.ticket), int(timeout_ms))
            if rc == L.IXB_ERR_TIMEOUT:
                raise TimeoutError(f"submitted run {self.ticket} did not complete within {timeout_ms} ms")
            L.check(rc)
            ms = C.c_float()
            self._s.lib.ixb_session_last_ms(self._s._h, C.byref(ms))
            self.gpu_ms = float(ms.value)
            self._result = self._egress
            self._keep = None
        return self._result

    def _retire(self) -> None:
        """Complete the run and detach its result from the slot buffer about to be reused."""
        out = self.wait(60000)
        if self._s._owns(out):
            self._result = out.copy()


class DetectHandle:
    """One submitted detection run in flight: the reference's ``ignite_run_async`` ticket
    (c_api/ignite.h:102-124). ``wait`` blocks until the detections are in host memory and
    returns one ``Detections`` per image (copied out of the session's pinned slot)."""

    def __init__(self, session: "GraphSession", ticket: int, batch: int, keep: Any):
        self._s = session
        self.ticket = int(ticket)
        self.batch = int(batch)
        self._keep = keep
        self._result = None
        self._error: Optional[Exception] = None

    @property
    def done(self) -> bool:
        return self._result is not None or self._error is not None

    @staticmethod
    def _view(ptr: int, dtype, shape):
        """A numpy view of the session's pinned detections (no copy)."""
        n = int(np.prod(shape))
        ct = {np.float32: C.c_float, np.int32: C.c_int32}[dtype]
        return np.frombuffer((ct * max(n, 1)).from_address(ptr), dtype=dtype, count=n).reshape(shape)

    def wait(self, timeout_ms: int = 2000):
        from .decode import Detections
        if self._error is not None:
            raise self._error
        if self._result is None:
            s = self._s
            n = C.c_int32()
            ptrs = [C.c_void_p() for _ in range(4)]
            rc = s.lib.ixb_session_detections(s._h, C.c_uint64(self.ticket), int(timeout_ms), C.byref(n),
                                              *[C.byref(p) for p in ptrs])
            if rc == L.IXB_ERR_TIMEOUT:
                raise TimeoutError(f"submitted run {self.ticket} did not complete within {timeout_ms} ms")
            L.check(rc)
            b, cap = int(n.value), s._det_capacity
            counts = self._view(ptrs[0].value, np.int32, (b,)).copy()
            boxes = self._view(ptrs[1].value, np.float32, (b, cap, 4))
            scores = self._view(ptrs[2].value, np.float32, (b, cap))
            classes = self._view(ptrs[3].value, np.int32, (b, cap))
            self._keep = None
            over = [i for i in range(b) if counts[i] < 0]
            if over:
                self._error = RuntimeError(f"image {over[0]}: more than {cap} detections survive NMS")
                raise self._error
            self._result = [Detections(boxes[i, :k].copy(), scores[i, :k].copy(), classes[i, :k].copy())
                            for i, k in enumerate(int(c) for c in counts)]
        return self._result

    def _retire(self) -> None:
        """Complete the run and copy its detections out of the slot about to be reused; a failed
        run keeps its error for its own wait."""
        try:
            self.wait(60000)
        except RuntimeError:
            if self._error is None:
                raise


class GraphSession:
    """Whole-network XINT8 YOLOv8 on one B200: persistent arena, one CUDA graph per batch size."""

    def __init__(self, ir: GraphIR, device_index: int = 0, max_batch: int = 64, pipeline_depth: int = 3):
        torch = _torch()
        if not torch.cuda.is_available():
            raise RuntimeError("GraphSession needs a CUDA device; this engine has no CPU path")
        self.lib = L.load()
        self.ir = ir
        self.device_index = int(device_index)
        self.device = torch.device("cuda", self.device_index)
        self.max_batch = int(max_batch)
        self.plan: DevicePlan = build_plan(ir, self.max_batch, pipeline_depth)
        self.arena = torch.zeros(self.plan.arena_bytes, dtype=torch.uint8, device=self.device)
        blob = torch.from_numpy(self.plan.const_blob)
        self.arena[self.plan.const_offset:self.plan.const_offset + blob.numel()].copy_(blob.to(self.device))
        torch.cuda.synchronize(self.device)
        self._cplan = c_plan(self.plan)
        h = C.c_void_p()
        L.check(self.lib.ixb_session_create(C.byref(self._cplan), self.device_index,
                                            C.c_void_p(self.arena.data_ptr()), self.plan.arena_bytes, C.byref(h)))
        self._h = h
        self.layout = layout_from_plan(self.plan)
        self.head_names = tuple(n for n, _ in self.plan.ir.outputs)
        self.in_image_bytes = 3 * self.plan.img_h * self.plan.img_w
        self.out_bytes = self.plan.egress_image_bytes
        self._egress = np.zeros((self.max_batch, self.out_bytes), dtype=np.int8)
        self._staged = 0
        self.last_dispatch_ms = 0.0
        self.last_host_ms = 0.0
        self._next_ticket = 1
        self.pipeline_depth = 1 + len(self.plan.extra_images_offsets)
        self._inflight = [None] * self.pipeline_depth     # RunHandle / DetectHandle per pipeline slot
        self._pin_in = [None] * self.pipeline_depth
        self._pin_out = [None] * self.pipeline_depth
        self._decoder = None
        self._det_capacity = 0

    # ------------------------------------------------------------------ status
    @property
    def head_status(self) -> HeadStatus:
        return HeadStatus(True, f"{len(self.head_names)} heads in the plan's egress, {self.out_bytes} bytes per image",
                          self.layout)

    @property
    def stream_handle(self) -> int:
        return int(self.lib.ixb_session_stream(self._h) or 0)

    def streams(self):
        """(compute, h2d, d2h) cudaStream_t handles as ints: the session's compute stream and the
        copy streams of ``run_async``."""
        c, h, d = C.c_void_p(), C.c_void_p(), C.c_void_p()
        L.check(self.lib.ixb_session_streams(self._h, C.byref(c), C.byref(h), C.byref(d)))
        return int(c.value or 0), int(h.value or 0), int(d.value or 0)

    def launches(self, batch: int) -> int:
        return L.check(self.lib.ixb_session_launches(self._h, int(batch)))

    # ------------------------------------------------------------------ frame
    def _as_pixels(self, x: Any):
        """uint8 pixels [B,3,H,W]; an int8 tensor is the preprocessor's (pixel - 128) convention."""
        torch = _torch()
        if isinstance(x, torch.Tensor):
            if x.dtype == torch.int8:
                x = (x.view(torch.uint8) ^ 0x80)
            elif x.dtype != torch.uint8:
                raise TypeError(f"images must be uint8 pixels or int8 (pixel - 128), got {x.dtype}")
            if x.dim() == 3:
                x = x.unsqueeze(0)
            return x.contiguous()
        a = np.asarray(x)
        if a.dtype == np.int8:
            a = a.view(np.uint8) ^ np.uint8(0x80)
        elif a.dtype != np.uint8:
            raise TypeError(f"images must be uint8 pixels or int8 (pixel - 128), got {a.dtype}")
        if a.ndim == 3:
            a = a[None]
        return np.ascontiguousarray(a)

    def _check_shape(self, shape) -> int:
        if len(shape) != 4 or tuple(shape[1:]) != (3, self.plan.img_h, self.plan.img_w):
            raise ValueError(f"expected images [B, 3, {self.plan.img_h}, {self.plan.img_w}], got {tuple(shape)}")
        b = int(shape[0])
        if not 1 <= b <= self.max_batch:
            raise ValueError(f"batch {b} outside [1, {self.max_batch}]")
        return b

    def stage_input(self, input_tensor: Any) -> None:
        """Copy a batch of images into the device staging buffer (no compute)."""
        torch = _torch()
        self._drain()
        x = self._as_pixels(input_tensor)
        b = self._check_shape(x.shape)
        n = b * self.in_image_bytes
        dst = self.arena[self.plan.images_offset:self.plan.images_offset + n]
        if isinstance(x, torch.Tensor):
            dst.copy_(x.reshape(-1).to(self.device))
        else:
            dst.copy_(torch.from_numpy(x.reshape(-1)).to(self.device))
        torch.cuda.synchronize(self.device)
        self._staged = b
        self._staged_store = False

    # ------------------------------------------------------------------ pipelined runs
    def _owns(self, a: np.ndarray) -> bool:
        for t in self._pin_out:
            if t is not None and np.shares_memory(a, t.numpy()):
                return True
        return False

    def _drain(self) -> None:
        for h in self._inflight:
            if h is not None and not h.done:
                h._retire()
        self._inflight = [None] * self.pipeline_depth

    def run_async(self, input_tensor: Any, unswizzle: bool = True, out: Optional[np.ndarray] = None,
                  detect: bool = False, letterbox: Optional[np.ndarray] = None):
        """Submit a batch and return at once (the reference's ``InferenceSession.run_async``,
        runtime/session.py:1280-1318).

        The images' host-to-device copy, the network and the heads' device-to-host copy run on
        three streams ordered by events, and consecutive submits rotate through
        ``pipeline_depth`` staging and egress slots (three by default), so one batch's H2D copy,
        another's compute and a third's D2H copy proceed together. ``input_tensor``
        is as for ``run``; a pinned CPU or a CUDA tensor is copied from in place (and must not be
        changed until the handle completes), anything else is first copied into the slot's pinned
        staging buffer. ``out``, if given, is an int8 [>=B, egress_image_bytes] array (pinned for
        overlap) that receives the heads; ``unswizzle`` is accepted for compatibility.

        ``detect=True`` (after ``set_detect``) appends the GPU decode + NMS to the run and brings back
        only the detections (a ``DetectHandle``; ``letterbox`` float [B, 3] maps boxes back to source
        pixels) instead of the heads: the reference's ``ignite_run_async`` contract."""
        torch = _torch()
        x = self._as_pixels(input_tensor)
        b = self._check_shape(x.shape)
        slot = (self._next_ticket - 1) % self.pipeline_depth
        prev = self._inflight[slot]
        if prev is not None and not prev.done:
            prev._retire()
        n = b * self.in_image_bytes
        if isinstance(x, torch.Tensor) and (x.is_cuda or x.is_pinned()):
            if x.is_cuda:
                torch.cuda.current_stream(x.device).synchronize()
            src, keep = x, x
        else:
            if self._pin_in[slot] is None:
                self._pin_in[slot] = torch.empty(self.max_batch * self.in_image_bytes, dtype=torch.uint8,
                                                 pin_memory=True)
            buf = self._pin_in[slot]
            host = x if isinstance(x, torch.Tensor) else torch.from_numpy(x)
            buf[:n].copy_(host.reshape(-1))
            src, keep = buf, None
        if detect:
            if self._decoder is None:
                raise RuntimeError("call set_detect() before detection runs")
            lb = None
            if letterbox is not None:
                lb = np.ascontiguousarray(np.asarray(letterbox, dtype=np.float32).reshape(b, 3))
            ticket = C.c_uint64()
            L.check(self.lib.ixb_session_submit_detect(self._h, C.c_void_p(src.data_ptr()), b,
                                                       lb.ctypes.data_as(C.c_void_p) if lb is not None else None,
                                                       C.byref(ticket)))
            return self._track(DetectHandle(self, ticket.value, b, keep), slot, b)
        if out is None:
            if self._pin_out[slot] is None:
                self._pin_out[slot] = torch.empty((self.max_batch, self.out_bytes), dtype=torch.int8,
                                                  pin_memory=True)
            egress = self._pin_out[slot].numpy()[:b]
        else:
            egress = out
            if egress.dtype != np.int8 or not egress.flags.c_contiguous or egress.size < b * self.out_bytes:
                raise ValueError(f"out must be a contiguous int8 array of at least {b} x {self.out_bytes}")
            egress = egress.reshape(-1)[:b * self.out_bytes].reshape(b, self.out_bytes)
        ticket = C.c_uint64()
        L.check(self.lib.ixb_session_submit(self._h, C.c_void_p(src.data_ptr()), b,
                                            egress.ctypes.data_as(C.c_void_p), C.byref(ticket)))
        return self._track(RunHandle(self, ticket.value, b, egress, keep), slot, b)

    def _track(self, h, slot: int, b: int):
        if h.ticket != self._next_ticket:
            raise RuntimeError(f"engine issued ticket {h.ticket}, expected {self._next_ticket}")
        self._next_ticket += 1
        self._inflight[slot] = h
        self._last_batch = b
        return h

    # ------------------------------------------------------------------ detection stage
    def set_detect(self, conf: float = 0.25, iou: float = 0.50, capacity: int = 300, class_names=None) -> None:
        """Attach the GPU decode + NMS stage (the reference's ``ignite_set_thresholds``, c_api/ignite.h:141,
        and its post-processing worker, ignite.cpp:640-980): detection runs bring back at most ``capacity``
        detections per image instead of the heads."""
        from .decode import GpuDecoder
        self._drain()
        dec = GpuDecoder(self.layout, self.plan.img_w, self.device, conf=conf, iou=iou)
        cfg = dec.config(capacity)
        L.check(self.lib.ixb_session_set_detect(self._h, C.byref(cfg)))
        self._decoder, self._det_cfg, self._det_capacity = dec, cfg, int(capacity)
        if class_names is not None:
            names = [str(n).encode() for n in class_names]
            arr = (C.c_char_p * len(names))(*names)
            L.check(self.lib.ixb_session_set_class_names(self._h, arr, len(names)))

    def set_thresholds(self, conf: float, iou: float) -> None:
        """Change the decode thresholds of the detection stage (``ignite_set_thresholds``)."""
        if self._decoder is None:
            raise RuntimeError("call set_detect() first")
        self._drain()
        L.check(self.lib.ixb_session_set_thresholds(self._h, float(conf), float(iou)))

    def submit_frames(self, frames: Any) -> DetectHandle:
        """uint8 BGR frames [B, H, W, 3] (host or CUDA, all one size): copied in, letterboxed and quantized
        on the GPU, run through the network, decoded on the GPU; the detections come back in source
        pixels (the reference's ``ignite_run_async`` on a batch)."""
        torch = _torch()
        if self._decoder is None:
            raise RuntimeError("call set_detect() before detection runs")
        if isinstance(frames, torch.Tensor):
            x = frames.contiguous()
        else:
            x = torch.from_numpy(np.ascontiguousarray(frames))
        if x.dtype != torch.uint8 or x.dim() != 4 or x.shape[3] != 3:
            raise ValueError(f"expected uint8 BGR frames [B, H, W, 3], got {tuple(x.shape)} {x.dtype}")
        b, h, w = int(x.shape[0]), int(x.shape[1]), int(x.shape[2])
        if not 1 <= b <= self.max_batch:
            raise ValueError(f"batch {b} outside [1, {self.max_batch}]")
        slot = (self._next_ticket - 1) % self.pipeline_depth
        prev = self._inflight[slot]
        if prev is not None and not prev.done:
            prev._retire()
        if x.is_cuda:
            torch.cuda.current_stream(x.device).synchronize()
        ticket = C.c_uint64()
        L.check(self.lib.ixb_session_submit_frames(self._h, C.c_void_p(x.data_ptr()), b, w, h, 3 * w, 3 * w * h,
                                                   C.byref(ticket)))
        return self._track(DetectHandle(self, ticket.value, b, x), slot, b)

    def run_frame(self, img_bgr: Any, max_detections: int = 300):
        """One BGR frame [H, W, 3] to detections, synchronously: the reference's ``ignite_run``
        (c_api/ignite.h:80-88) through the C ABI's ``ixb_run_frame``. Returns a list of
        (x0, y0, w, h, score, class_id, class_name)."""
        if self._decoder is None:
            raise RuntimeError("call set_detect() before detection runs")
        self._drain()
        a = np.ascontiguousarray(img_bgr, dtype=np.uint8)
        if a.ndim != 3 or a.shape[2] != 3:
            raise ValueError(f"expected a BGR frame [H, W, 3], got {a.shape}")
        out = (L.Detection * max(1, int(max_detections)))()
        n = L.check(self.lib.ixb_run_frame(self._h, a.ctypes.data_as(C.c_void_p), a.shape[1], a.shape[0],
                                           3 * a.shape[1], out, int(max_detections)))
        self._next_ticket += 1          # the engine's ticket of that run
        return [(d.x0, d.y0, d.w, d.h, d.score, d.class_id, d.class_name.decode()) for d in out[:n]]

    @property
    def last_timings(self) -> Dict[str, float]:
        """Stages of the last completed detection run (the reference's ``ignite_get_last_timings``)."""
        t = L.Timings()
        L.check(self.lib.ixb_session_last_timings(self._h, C.byref(t)))
        return {k: float(getattr(t, k)) for k, _ in L.Timings._fields_}

    def decode_predictions(self, batch: Optional[int] = None):
        """The dense decode of the heads in the device egress, on the GPU: float32 CUDA tensor
        [B, 84, anchors] (the reference's ``decode_yolo_predictions``, runtime/session.py:1223-1278)."""
        from .decode import dense_heads
        torch = _torch()
        b = int(batch or getattr(self, "_last_batch", self._staged) or 1)
        heads = dense_heads(self.layout, self.plan.img_w)
        total = sum(int(h.grid) ** 2 for h in heads)
        out = torch.empty((b, 4 + 80, total), dtype=torch.float32, device=self.device)
        eg = self.arena[self.plan.egress_offset:self.plan.egress_offset + b * self.out_bytes]
        L.check(self.lib.ixb_decode_dense(heads, 80, C.c_void_p(eg.data_ptr()), b, self.out_bytes,
                                          C.c_void_p(out.data_ptr()), C.c_void_p(self.stream_handle)))
        torch.cuda.synchronize(self.device)
        return out


    def stage_image(self, img_bgr: Any):
        """Letterbox, resize and quantize one BGR frame into the stem's input on the device (the
        reference's ``GraphSession.stage_image``, graph_session.py:866-889); returns the letterbox
        ``((pad_top, pad_left), scale)`` for box decoding."""
        lb = self.stage_images(img_bgr[None])
        return (int(lb[0, 0]), int(lb[0, 1])), float(lb[0, 2])

    def stage_images(self, frames: Any) -> np.ndarray:
        """uint8 BGR frames [B, H, W, 3] (host or CUDA, all one size) -> letterboxed into the stem's
        input by the GPU kernel; returns float32 [B, 3] (pad_top, pad_left, scale) per image."""
        torch = _torch()
        self._drain()
        x = frames if isinstance(frames, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(frames))
        if x.dtype != torch.uint8 or x.dim() != 4 or x.shape[3] != 3:
            raise ValueError(f"expected uint8 BGR frames [B, H, W, 3], got {tuple(x.shape)} {x.dtype}")
        b = int(x.shape[0])
        if not 1 <= b <= self.max_batch:
            raise ValueError(f"batch {b} outside [1, {self.max_batch}]")
        x = x.contiguous().to(self.device)
        h, w = int(x.shape[1]), int(x.shape[2])
        lb = (C.c_float * 3)()
        L.check(self.lib.ixb_session_letterbox(self._h, C.c_void_p(x.data_ptr()), b, w, h, 3 * w, 3 * w * h, lb))
        torch.cuda.synchronize(self.device)
        self._staged = b
        self._staged_store = True
        return np.tile(np.array(list(lb), dtype=np.float32), (b, 1))

    def dispatch(self, timeout_ms: int = 10000, batch: Optional[int] = None) -> None:
        """Run the network on the staged images; heads stay in the device egress."""
        self._drain()
        b = int(batch or self._staged)
        if b < 1:
            raise RuntimeError("no staged input")
        src = L.IN_STORE if getattr(self, "_staged_store", False) else L.IN_DEVICE
        L.check(self.lib.ixb_session_run(self._h, None, b, None, src | L.OUT_DEVICE | L.ASYNC))
        self._wait(timeout_ms)
        self._last_batch = b

    def _wait(self, timeout_ms: int) -> None:
        rc = self.lib.ixb_session_wait(self._h, int(timeout_ms))
        if rc == L.IXB_ERR_TIMEOUT:
            raise TimeoutError(f"GPU dispatch did not complete within {timeout_ms} ms")
        L.check(rc)
        ms = C.c_float()
        self.lib.ixb_session_last_ms(self._h, C.byref(ms))
        self.last_dispatch_ms = float(ms.value)

    def read_heads(self, unswizzle: bool = True, batch: Optional[int] = None) -> np.ndarray:
        """Copy the int8 NCHW egress [B, bytes] back to the host."""
        torch = _torch()
        b = int(batch or getattr(self, "_last_batch", self._staged) or 1)
        src = self.arena[self.plan.egress_offset:self.plan.egress_offset + b * self.out_bytes]
        out = src.cpu().numpy().view(np.int8).reshape(b, self.out_bytes)
        self._egress[:b] = out
        return self._egress[:b]

    def run_yolo_monolithic(self, input_tensor: Any, unswizzle: bool = True, timeout_ms: int = 10000,
                            return_timestamps: bool = False, max_segments: Optional[int] = None):
        """Whole-network forward pass of a batch; the reference's head dictionary with a batch dimension.

        ``input_tensor`` is uint8 pixels [B,3,H,W] (or [3,H,W]) or the int8 (pixel - 128) tensor of the
        reference's preprocessor, host or CUDA memory; ``None`` runs the images staged by ``stage_input``.
        ``unswizzle`` and ``max_segments`` are accepted for compatibility: the heads are always NCHW
        and the network is one segment."""
        torch = _torch()
        self._drain()
        t0 = time.perf_counter()
        if input_tensor is None:
            b = self._staged
            if b < 1:
                raise RuntimeError("no staged input")
            src = L.IN_STORE if getattr(self, "_staged_store", False) else L.IN_DEVICE
            L.check(self.lib.ixb_session_run(self._h, None, b, None, src | L.OUT_DEVICE | L.ASYNC))
        else:
            x = self._as_pixels(input_tensor)
            b = self._check_shape(x.shape)
            if isinstance(x, torch.Tensor) and x.is_cuda:
                torch.cuda.current_stream(x.device).synchronize()
                L.check(self.lib.ixb_session_run(self._h, C.c_void_p(x.data_ptr()), b,
                                                 self._egress.ctypes.data_as(C.c_void_p), L.IN_DEVICE | L.ASYNC))
            else:
                if isinstance(x, torch.Tensor):
                    x = x.numpy()
                L.check(self.lib.ixb_session_run(self._h, x.ctypes.data_as(C.c_void_p), b,
                                                 self._egress.ctypes.data_as(C.c_void_p), L.ASYNC))
        t1 = time.perf_counter()
        self._wait(timeout_ms)
        t2 = time.perf_counter()
        self._last_batch = b
        egress = self.read_heads(batch=b) if input_tensor is None else self._egress[:b]
        t3 = time.perf_counter()
        out: Dict[str, Any] = dict(self.layout.unpack(egress))
        out["scales"] = self.layout.scales()
        out["heads_present"] = True
        out["head_status"] = self.head_status.reason
        out["raw_output"] = egress
        out["raw_heads"] = egress
        out["unswizzled"] = True
        if return_timestamps:
            ts = {"stage_ms": (t1 - t0) * 1e3, "npu_ms": self.last_dispatch_ms, "gpu_ms": self.last_dispatch_ms,
                  "host_ms": 0.0, "readback_ms": (t3 - t2) * 1e3, "wall_ms": (t3 - t0) * 1e3}
            return out, ts
        return out

    def run(self, input_tensor: Any, **kwargs) -> np.ndarray:
        return self.run_yolo_monolithic(input_tensor, **kwargs)["raw_output"]

    # ------------------------------------------------------------------ parity helpers
    def read_tensor(self, name: str, batch: Optional[int] = None) -> np.ndarray:
        """A stored activation as the reference holds it: uint8 (zero point 128) [B, C, H, W]."""
        b = int(batch or getattr(self, "_last_batch", 1))
        if name in dict((t, n) for n, t in self.ir.outputs):
            head = [n for n, t in self.ir.outputs if t == name][0]
            h = self.layout.unpack(self.read_heads(batch=b))[head]
            return (h.astype(np.int16) + 128).astype(np.uint8)
        if name == self.ir.input and self.plan.input_s2d_store is not None:
            v = self._read_store(self.plan.input_s2d_store, b)     # [b, 16, H/2, W/2], byte ph * 3 + c
            out = np.empty((b, 3, 2 * v.shape[2], 2 * v.shape[3]), dtype=np.uint8)
            for ph in range(4):
                ry, rx = divmod(ph, 2)
                out[:, :, ry::2, rx::2] = v[:, 3 * ph:3 * ph + 3]
            return out
        if name == self.ir.input:
            st = self.plan.input_store
            raw = self.arena[st.offset:st.offset + b * (st.height + 2) * (st.width + 4) * 8].cpu().numpy()
            v = raw.view(np.int8).reshape(b, st.height + 2, st.width + 4, 8)[:, 1:-1, 1:st.width + 1, :3]
            return (v.astype(np.int16) + 128).astype(np.uint8).transpose(0, 3, 1, 2)
        if name in self.plan.s2d_only:
            # stored only as its space-to-depth view: phase (ry, rx) = divmod(chunk group, 2)
            v = self._read_store(self.plan.s2d_stores[name], b)
            n = v.shape[1] // 4
            t = self.ir.tensors[name]
            out = np.empty((b, n, 2 * v.shape[2], 2 * v.shape[3]), dtype=np.uint8)
            for ph in range(4):
                ry, rx = divmod(ph, 2)
                out[:, :, ry::2, rx::2] = v[:, ph * n:(ph + 1) * n]
            return out[:, :t.channels]
        return self._read_store(self.plan.stores[name], b)[:, :self.ir.tensors[name].channels]

    def _read_store(self, st, b: int) -> np.ndarray:
        """uint8 [b, channels, H, W] of one stored tensor (the halo ring dropped)."""
        P = (st.height + 2) * (st.width + 2)
        out = np.empty((b, st.channels, st.height, st.width), dtype=np.uint8)
        for c in range(st.channels // 16):
            o = st.offset + (st.chunk_offset + c) * st.plane_stride
            raw = self.arena[o:o + b * P * 16].cpu().numpy().view(np.int8).reshape(b, st.height + 2, st.width + 2, 16)
            v = raw[:, 1:-1, 1:-1, :].transpose(0, 3, 1, 2)
            out[:, 16 * c:16 * c + 16] = (v.astype(np.int16) + 128).astype(np.uint8)
        return out     # stored zero channels past a ragged tail are sliced off by the caller

    def trace(self, batch: int, iters: int = 3):
        """Device timeline of a graph run: per op (start, inputs ready, end) in microseconds from the
        first op's start, as the ops execute in the graph (pool ops: None)."""
        self._drain()
        n = len(self.plan.ops)
        ns = (C.c_uint64 * (3 * n))()
        L.check(self.lib.ixb_session_trace(self._h, int(batch), int(iters), ns))
        v = np.array(ns[:], dtype=np.int64).reshape(n, 3)
        t0 = v[v[:, 0] > 0, 0].min()
        return [None if r[0] == 0 else tuple((r - t0) / 1000.0) for r in v]

    def profile(self, batch: int, iters: int = 3):
        """Mean device milliseconds per op (layer-by-layer launches with events)."""
        self._drain()
        ms = (C.c_float * len(self.plan.ops))()
        L.check(self.lib.ixb_session_profile(self._h, int(batch), int(iters), ms))
        return list(ms)

    # ------------------------------------------------------------------ lifetime
    def close(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                self._drain()
            except Exception:
                pass
            self.lib.ixb_session_destroy(h)
            self._h = C.c_void_p()
        self.arena = None

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        self.close()
        return False

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def decode_yolo_predictions(head_outputs: Dict[str, np.ndarray], strides=(8, 16, 32)) -> np.ndarray:
        return InferenceSession.decode_yolo_predictions(head_outputs, strides)


class InferenceSession:
    """Entry points of the reference's ``ignite_xdna.InferenceSession`` that serve this path."""

    @classmethod
    def from_spec(cls, model: str = "yolov8n", seed: int = 0, imgsz: int = 640, device_index: int = 0,
                  max_batch: int = 64, pipeline_depth: int = 3, **kw) -> GraphSession:
        """Open a session on the seeded synthetic XINT8 graph ``model`` in {yolov8n, yolov8s, yolov8m},
        or their YOLOv8-pose versions ``yolov8n-pose`` ... (nine heads: one class plus keypoints)."""
        from .yolov8 import build_yolov8
        variant = model.replace("yolov8", "")
        if variant.endswith("-pose"):
            variant = variant[:-len("-pose")]
            kw["task"] = "pose"
        return GraphSession(build_yolov8(variant, imgsz=imgsz, seed=seed, **kw), device_index=device_index,
                            max_batch=max_batch, pipeline_depth=pipeline_depth)

    @classmethod
    def from_file(cls, path: Union[str, Path], device_index: int = 0, max_batch: int = 64, **kwargs) -> GraphSession:
        """Open an ``.ignite`` container holding a quantized graph (``container.save_container``), a
        pickled ``GraphIR`` (as ``save_graph`` writes), or a ``yolov8{n,s,m}[_<imgsz>]`` spec name
        (the reference's ``InferenceSession.from_file``, runtime/session.py:1496)."""
        p = Path(path)
        if p.exists():
            with open(p, "rb") as f:
                magic = f.read(4)
            if magic == b"IGNT":
                from .container import load_container
                return GraphSession(load_container(p), device_index=device_index, max_batch=max_batch)
            import pickle
            with open(p, "rb") as f:
                ir = pickle.load(f)
            if not isinstance(ir, GraphIR):
                raise ValueError(f"{p} does not hold a GraphIR")
            return GraphSession(ir, device_index=device_index, max_batch=max_batch)
        name = p.name
        if name.startswith("yolov8"):
            parts = name.split("_")
            imgsz = int(parts[1]) if len(parts) > 1 else 640
            return cls.from_spec(parts[0], imgsz=imgsz, device_index=device_index, max_batch=max_batch, **kwargs)
        raise FileNotFoundError(path)

    @staticmethod
    def decode_yolo_predictions(head_outputs: Dict[str, np.ndarray], strides=(8, 16, 32)) -> np.ndarray:
        """Heads -> [B, 84, anchors]: DFL softmax + integral over 16 bins, dist2bbox xywh, class sigmoid
        (runtime/session.py:1223-1278), in float32 numpy."""
        scales = head_outputs.get("scales")

        def as_float(name):
            t = head_outputs.get(name)
            if t is None:
                return None
            if t.dtype == np.int8:
                s, zp = scales[name]
                return (t.astype(np.float32) - np.float32(zp)) * np.float32(s)
            return t

        preds = []
        bins = np.arange(16, dtype=np.float32)
        for lvl, stride in zip((3, 4, 5), strides):
            box, cls = as_float(f"p{lvl}_box"), as_float(f"p{lvl}_cls")
            if box is None or cls is None:
                continue
            if box.ndim == 3:
                box, cls = box[None], cls[None]
            b, _, h, w = box.shape
            bf = box.reshape(b, 4, 16, h * w)
            e = np.exp(bf - bf.max(axis=2, keepdims=True))
            dist = (e / e.sum(axis=2, keepdims=True) * bins[None, None, :, None]).sum(axis=2)
            yv, xv = np.meshgrid(np.arange(h, dtype=np.float32), np.arange(w, dtype=np.float32), indexing="ij")
            gx, gy = xv.reshape(-1), yv.reshape(-1)
            x1 = (gx - dist[:, 0]) * stride
            y1 = (gy - dist[:, 1]) * stride
            x2 = (gx + dist[:, 2]) * stride
            y2 = (gy + dist[:, 3]) * stride
            xywh = np.stack([(x1 + x2) / 2, (y1 + y2) / 2, x2 - x1, y2 - y1], axis=1)
            prob = 1.0 / (1.0 + np.exp(-cls.reshape(b, cls.shape[1], h * w)))
            preds.append(np.concatenate([xywh, prob], axis=1))
        return np.concatenate(preds, axis=2) if preds else np.zeros((1, 84, 8400), dtype=np.float32)


def save_graph(ir: GraphIR, path: Union[str, Path]) -> None:
    """Write ``ir`` as an ``.ignite`` container (a path ending in .ignite) or a pickle."""
    if str(path).endswith(".ignite"):
        from .container import save_container
        save_container(ir, path, model_name=Path(path).stem)
        return
    import pickle
    with open(path, "wb") as f:
        pickle.dump(ir, f)
