"""Benchmark: XINT8 YOLOv8n images/sec on 1..8 B200 (batch 64 per GPU, 640x640), one replica per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--model yolov8n] [--batch 64]
    python bench.py --impl reference ...     # the CPU integer reference on the host cores

One JSON line on rank 0. A step is one pass of the whole network over one batch of 64
seeded uniform-uint8 images per GPU. ``value`` times K steps with the images already in HBM
(CUDA events on the session's stream, max over ranks, barrier + synchronize on both sides);
``e2e`` times K steps through the public API (``GraphSession.run_async(detect=True)``, the
reference's ignite_run contract) from pinned host images to pinned host detections, both copies of
every step inside the timed region; ``e2e_heads`` does the same with the raw int8 heads coming
back instead (``GraphSession.run_async``). Multi-GPU runs are independent replicas:
each rank owns its GPU, its weights and its images; there is no collective on the data path
(the process group only carries the barrier and the max of the timings).
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "YOLOv8n int8 images/sec at 1/2/4/8 B200 (bs64/GPU, 640²); % int8 TC peak"
UNIT = "images/s"
L2_BYTES = 126 * 1024 * 1024
DET_CAPACITY = 8400   # detections kept per image by the e2e detection stage: every anchor


# ---------------------------------------------------------------- CPU baseline (oracle port)
_WORK_IR = None


def _cpu_init(ir):
    global _WORK_IR
    _WORK_IR = ir


def _cpu_one(seed_imgsz):
    sys.path.insert(0, str(ROOT / "oracle"))
    import ixb_oracle as O
    from ignite_xdna_b200 import random_images
    seed, imgsz = seed_imgsz
    t = O.run_image(_WORK_IR, random_images(1, imgsz, seed=seed)[0])
    return len(t)


def cpu_pool(ir, cores):
    env_keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    saved = {k: os.environ.get(k) for k in env_keys}
    for k in env_keys:
        os.environ[k] = "1"
    try:
        pool = mp.get_context("spawn").Pool(cores, initializer=_cpu_init, initargs=(ir,))
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return pool


def cpu_images_per_sec(pool, n_images, imgsz, seed0=1000):
    t0 = time.perf_counter()
    pool.map(_cpu_one, [(seed0 + i, imgsz) for i in range(n_images)], chunksize=1)
    return n_images / (time.perf_counter() - t0)


def cpu_baseline(ir, imgsz, cores):
    pool = cpu_pool(ir, cores)
    try:
        pool.map(_cpu_one, [(999, imgsz)] * cores, chunksize=1)       # workers import numpy, warm up
        n = max(8, 2 * cores)
        v = cpu_images_per_sec(pool, n, imgsz)
    finally:
        pool.close()
        pool.join()
    return {"value": round(v, 3), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} images of the same workload through oracle/ixb_oracle.run_image (numpy restatement "
                      f"of the reference's graph_reference.run_direct), one image per worker process, "
                      f"{cores} single-threaded workers"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and throttle reasons sampled DURING the timed region: NVML every 5 ms in a thread
    (the timed region lasts tens of milliseconds), else ``nvidia-smi -lms 100``. Reads only."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, device_index):
        self.dev = device_index
        self.rows = []          # (sm_mhz, max_mhz, set of reasons)
        self.proc = None
        self.nvml = None
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        pr = torch.cuda.get_device_properties(self.dev)
        try:
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def __enter__(self):
        try:
            self.nvml, h = self._nvml_handle()
            mx = self.nvml.nvmlDeviceGetMaxClockInfo(h, self.nvml.NVML_CLOCK_SM)

            def poll():
                while not self.stop.is_set():
                    try:
                        mhz = self.nvml.nvmlDeviceGetClockInfo(h, self.nvml.NVML_CLOCK_SM)
                        bits = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:
                        break
                    self.rows.append((float(mhz), float(mx), {n for n, b in self.REASONS.items() if bits & b}))
                    self.stop.wait(0.005)
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.proc.stdout:
            r = [x.strip() for x in line.split(",")]
            try:
                self.rows.append((float(r[1]), float(r[2]),
                                  {n for n, v in zip(names, r[5:9]) if v.lower().startswith("active")}))
            except (ValueError, IndexError):
                continue

    def __exit__(self, *a):
        self.stop.set()
        if self.nvml is not None:
            self.t.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set().union(*(r[2] for r in self.rows))
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.rows[-1][1],
                "reasons": sorted(reasons), "samples": len(self.rows),
                "source": "nvml 5 ms" if self.nvml is not None else "nvidia-smi 100 ms"}


# ---------------------------------------------------------------- helpers
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def bind_to_gpu_numa(local):
    """Run this rank's host threads, and so place its pinned buffers (first touch), on the NUMA node
    its GPU hangs off (sysfs: the PCI device's numa_node and that node's cpulist), so that host <->
    device copies do not cross the socket link. Returns the node, or None where sysfs does not say."""
    try:
        import torch
        pr = torch.cuda.get_device_properties(local)
        pci = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{pci}/numa_node").read_text().strip())
        if node < 0:
            return None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, local):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def layer_algorithmic(ir, L, batch):
    """Algorithmic bytes and int8 ops of one conv launch: every input activation read once, the
    output (and a residual) once, the weights and bias once; 2 ops per MAC."""
    t = ir.tensors[L.output]
    nbytes = 0
    for s in L.inputs:
        src = ir.tensors[s.tensor]
        if s.tensor == ir.input:
            nbytes += batch * 3 * src.height * src.width
        else:
            nbytes += batch * s.blocks * 8 * src.height * src.width
    if L.residual is not None:
        nbytes += batch * L.cout * t.height * t.width
    nbytes += batch * L.cout * t.height * t.width + L.weights.size + 4 * L.cout
    ops = 2 * batch * t.height * t.width * L.cout * L.cin * L.k * L.k
    return nbytes, ops


def conv_algorithmic(ir, batch):
    """Per-step algorithmic bytes and int8 ops of all conv launches."""
    nbytes = ops = 0
    for L in ir.conv_layers():
        b, o = layer_algorithmic(ir, L, batch)
        nbytes += b
        ops += o
    return nbytes, ops


def per_layer_rows(sess, batch, trace, int8_peak_tops):
    """One row per conv op from the in-graph trace (ready -> end, under programmatic dependent launch
    and in the step's own order): microseconds, int8 TOP/s, tensor fraction, algorithmic GB/s."""
    from ignite_xdna_b200 import _lib as L
    rows = []
    group, members = -1, {}
    for kind, _ in sess.plan.ops:  # an op flagged OP_WITH_PREV runs beside the ops before it
        if not kind & L.OP_WITH_PREV:
            group += 1
        members[group] = members.get(group, 0) + 1
    group = -1
    for (kind, idx), t in zip(sess.plan.ops, trace):
        if not kind & L.OP_WITH_PREV:
            group += 1
        if (kind & 0xFF) != L.OP_CONV or t is None:
            continue
        layer = sess.plan.convs[idx].layer
        nbytes, ops = layer_algorithmic(sess.ir, layer, batch)
        us = max(t[2] - t[1], 1e-3)
        tops = ops / (us * 1e-6) / 1e12
        t_out = sess.ir.tensors[layer.output]
        rows.append({"op": idx, "layer": layer.name, "k": layer.k, "stride": layer.stride, "cin": layer.cin,
                     "cout": layer.cout, "out": f"{t_out.height}x{t_out.width}", "us": round(us, 2), "int8_tops": round(tops, 1),
                     "tc_frac": round(tops / int8_peak_tops, 4),
                     "gbs": round(nbytes / (us * 1e-6) / 1e9, 1), "group": group,
                     "concurrent_with": members[group] - 1})
    return rows


def busy_us(intervals):
    """Length of the union of [a, b] intervals: the time at least one of them runs."""
    total, cur = 0.0, None
    for a, b in sorted(intervals):
        if cur is None or a > cur[1]:
            if cur is not None:
                total += cur[1] - cur[0]
            cur = [a, b]
        else:
            cur[1] = max(cur[1], b)
    return total + (cur[1] - cur[0] if cur is not None else 0.0)


def copy_ceiling(B, in_bytes, out_bytes, world, local, iters=5):
    """Pure-copy calibration on every rank at once, no compute: one step's images (pinned host ->
    HBM) and heads (HBM -> pinned host), alone and together, each direction on its own stream.
    Returns aggregate GB/s over all ranks (bytes of all ranks / the slowest rank's time) and the
    e2e images/s these copies alone allow."""
    import torch
    dev = torch.device("cuda", local)
    s_h2d, s_d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    n_in, n_out = B * in_bytes, B * out_bytes
    host_in = torch.empty(n_in, dtype=torch.uint8, pin_memory=True)
    host_out = torch.empty(n_out, dtype=torch.uint8, pin_memory=True)
    dst_in = torch.empty(n_in, dtype=torch.uint8, device=dev)
    src_out = torch.zeros(n_out, dtype=torch.uint8, device=dev)

    def timed(h2d, d2h):
        barrier(world)
        torch.cuda.synchronize(local)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(s_h2d)
        ev[2].record(s_d2h)
        for _ in range(iters):
            if h2d:
                with torch.cuda.stream(s_h2d):
                    dst_in.copy_(host_in, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s_d2h):
                    host_out.copy_(src_out, non_blocking=True)
        ev[1].record(s_h2d)
        ev[3].record(s_d2h)
        torch.cuda.synchronize(local)
        ms = max(ev[0].elapsed_time(ev[1]) if h2d else 0.0, ev[2].elapsed_time(ev[3]) if d2h else 0.0)
        barrier(world)
        return max_over_ranks(ms, world, local) / iters

    timed(True, True)                                     # warm-up
    t_in, t_out, t_both = timed(True, False), timed(False, True), timed(True, True)
    torch.cuda.synchronize(local)
    gbs = lambda nb, ms: round(world * nb / (ms * 1e-3) / 1e9, 1)  # noqa: E731
    return {"h2d_gbs": gbs(n_in, t_in), "d2h_gbs": gbs(n_out, t_out),
            "both_ms_per_step": round(t_both, 4), "h2d_bytes_per_rank": int(n_in), "d2h_bytes_per_rank": int(n_out),
            "images_s_ceiling": round(world * B / (t_both * 1e-3), 1),
            "note": "pinned host <-> HBM copies only, every rank at once, one stream per direction; "
                    "images_s_ceiling = what the images-in + heads-out copies alone allow"}


# ---------------------------------------------------------------- arms
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from ignite_xdna_b200 import build_yolov8
    ir = build_yolov8(args.model.replace("yolov8", ""), imgsz=args.imgsz)
    cores = os.cpu_count() or 1
    pool = cpu_pool(ir, cores)
    try:
        pool.map(_cpu_one, [(999, args.imgsz)] * cores, chunksize=1)
        per_step = cores
        for w in range(args.warmup):
            cpu_images_per_sec(pool, per_step, args.imgsz, seed0=2000 + w * per_step)
        t0 = time.perf_counter()
        for s in range(args.steps):
            pool.map(_cpu_one, [(3000 + s * per_step + i, args.imgsz) for i in range(per_step)], chunksize=1)
        dt = time.perf_counter() - t0
    finally:
        pool.close()
        pool.join()
    v = per_step * args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
            "data": "synthetic", "config": workload_config(args),
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"each step {per_step} images (one per host core) through the numpy "
                                       f"restatement of graph_reference.run_direct (oracle/ixb_oracle.py); "
                                       f"the reference itself is Python and is not present on the GPU host"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args):
    return {"workload": f"{args.model} XINT8 whole network, {args.imgsz}x{args.imgsz} uint8 images uniform "
                        f"[0,255] (seeded), batch {args.batch} per GPU, one replica per GPU",
            "global_batch": args.batch * int(os.environ.get("WORLD_SIZE", "1")), "batch_per_gpu": args.batch,
            "imgsz": args.imgsz, "parallelism": f"replicas x{int(os.environ.get('WORLD_SIZE', '1'))} (no collective)",
            "l2": f"each step's working set (activations of {args.batch} images, >1 GB) exceeds the 126 MB L2, so "
                  f"every step starts cold"}


def run_gpu(args):
    import ctypes as C
    world, rank, local = dist_setup(args)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from ignite_xdna_b200 import build_yolov8
        ir0 = build_yolov8(args.model.replace("yolov8", ""), imgsz=args.imgsz)
        cpu = cpu_baseline(ir0, args.imgsz, os.cpu_count() or 1)    # pool spawned before any GPU call
    import numpy as np
    import torch
    from ignite_xdna_b200 import InferenceSession, random_images
    from ignite_xdna_b200 import _lib as L
    torch.cuda.set_device(local)
    numa = bind_to_gpu_numa(local)
    # four slots: the next batch's H2D is queued a full step before the stream reaches it, so the
    # host's wake-up and submit latency after a D2H completes stays off the copy engines' path
    sess = InferenceSession.from_spec(args.model, imgsz=args.imgsz, device_index=local, max_batch=args.batch,
                                      pipeline_depth=args.depth)
    lib = sess.lib
    B = args.batch
    imgs = random_images(B, args.imgsz, seed=100 + rank)
    pinned_in = torch.from_numpy(imgs).pin_memory()
    depth = sess.pipeline_depth
    pinned_out = [torch.empty((B, sess.out_bytes), dtype=torch.int8).pin_memory().numpy() for _ in range(depth)]
    sess.stage_input(imgs)
    dev = torch.device("cuda", local)
    h_compute, h_h2d, h_d2h = sess.streams()
    stream = torch.cuda.ExternalStream(h_compute, device=dev)
    s_h2d, s_d2h = torch.cuda.ExternalStream(h_h2d, device=dev), torch.cuda.ExternalStream(h_d2h, device=dev)

    def device_step():
        # enqueue only: consecutive steps queue on the session's stream (ixb_session_run stacks
        # asynchronous runs), so the GPU runs them back to back as a serving loop keeps it fed;
        # timed() waits for them after its end event
        L.check(lib.ixb_session_run(sess._h, None, B, None, L.IN_DEVICE | L.OUT_DEVICE | L.ASYNC))

    def device_done():
        L.check(lib.ixb_session_wait(sess._h, 60000))

    def e2e_steps(k, detect=False):
        """k batches through GraphSession.run_async: pinned images in, pinned heads out (or, with
        ``detect``, the GPU decode + NMS after the network and only the detections out), up to
        ``depth`` in flight, so step i+1's H2D and step i-1's D2H overlap step i's compute."""
        hs = []
        for i in range(k):
            if detect:
                hs.append(sess.run_async(pinned_in, detect=True))
            else:
                hs.append(sess.run_async(pinned_in, out=pinned_out[i % depth]))
            if len(hs) == depth:
                hs.pop(0).wait(60000)
        for h in hs:
            h.wait(60000)

    def timed_e2e(k, detect=False):
        barrier(world)
        torch.cuda.synchronize(local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_h2d)
        e2e_steps(k, detect)
        e1.record(s_d2h)
        e1.synchronize()
        torch.cuda.synchronize(local)
        barrier(world)
        return e0.elapsed_time(e1)

    def timed(step, k, done=None):
        barrier(world)
        torch.cuda.synchronize(local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            step()
        e1.record(stream)
        e1.synchronize()
        if done is not None:
            done()  # completes the queued runs (and reads the device error flag)
        torch.cuda.synchronize(local)
        barrier(world)
        return e0.elapsed_time(e1)

    # the detection stage (GPU decode + NMS; capacity = every anchor, so no image can overflow)
    sess.set_detect(conf=0.25, iou=0.50, capacity=DET_CAPACITY)
    for _ in range(args.warmup):
        device_step()
    device_done()
    e2e_steps(max(3, args.warmup))
    e2e_steps(max(3, args.warmup), detect=True)
    with ClockSampler(local) as clocks:     # over the three timed regions
        ms = timed(device_step, args.steps, device_done)
        ms_e2e = timed_e2e(args.steps)
        ms_e2e_det = timed_e2e(args.steps, detect=True)
    ms = max_over_ranks(ms, world, local)
    ms_e2e = max_over_ranks(ms_e2e, world, local)
    ms_e2e_det = max_over_ranks(ms_e2e_det, world, local)
    det_d2h = (B * 4 + 15) // 16 * 16 + B * DET_CAPACITY * 24
    ceiling = copy_ceiling(B, sess.in_image_bytes, sess.out_bytes, world, local)
    # per-layer device times inside the step's own CUDA graph (programmatic dependent launch on):
    # each conv from the moment its inputs were ready to its last CTA's end
    hbm_peak, bf16_peak, peak_kind = load_peaks()
    trace = sess.trace(B, iters=3)
    rows = per_layer_rows(sess, B, trace, 2 * bf16_peak)
    # branch-group members run at the same time: the step's conv time is the union of their intervals
    conv_ms = busy_us([(t[1], t[2]) for (kind, _), t in zip(sess.plan.ops, trace)
                       if t is not None and (kind & 0xFF) == L.OP_CONV]) * 1e-3
    span_ms = max(t[2] for t in trace if t is not None) * 1e-3
    nbytes, nops = conv_algorithmic(sess.ir, B)
    achieved_gbs = nbytes / (conv_ms * 1e-3) / 1e9
    int8_tops = nops / (conv_ms * 1e-3) / 1e12
    launches = sess.launches(B)
    if rank != 0:
        sess.close()
        import torch.distributed as dist
        dist.destroy_process_group()
        return 0
    value = world * B * args.steps / (ms * 1e-3)
    traffic = None
    tp = ROOT / "profiles" / "conv_traffic.json"
    if tp.exists():
        try:
            traffic = json.loads(tp.read_text()).get(f"{args.model}_{args.imgsz}_b{B}")
        except (ValueError, OSError):
            traffic = None
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (int32 accumulate)",
        "data": "synthetic (seeded uniform uint8 images; seeded kaiming weights, pow2-quantized)",
        "config": workload_config(args),
        # the headline end-to-end number is the reference's ignite_run contract: images in, detections
        # out (decode + NMS on the GPU); the heads path (raw int8 heads back) is reported beside it
        "e2e": {"value": round(world * B * args.steps / (ms_e2e_det * 1e-3), 1), "unit": UNIT,
                "ms_per_step": round(ms_e2e_det / args.steps, 4),
                "h2d_bytes_per_step": int(B * (sess.in_image_bytes + 12)), "d2h_bytes_per_step": int(det_d2h),
                "path": "GraphSession.run_async(detect=True) (C ABI ixb_session_submit_detect / "
                        "ixb_session_detections, the reference's ignite_run_async / ignite_wait contract): "
                        "pinned host images -> H2D stream -> graph + GPU decode/NMS (conf 0.25, iou 0.5) on the "
                        f"compute stream -> D2H of the detections (capacity {DET_CAPACITY} per image) -> pinned "
                        f"host, {depth} batches in flight; CUDA events from the first H2D to the last D2H; every "
                        "anchor of the synthetic graph passes the 0.25 prune, so the NMS sees 8400 candidates "
                        "per image"},
        "e2e_heads": {"value": round(world * B * args.steps / (ms_e2e * 1e-3), 1), "unit": UNIT,
                      "ms_per_step": round(ms_e2e / args.steps, 4),
                      "h2d_bytes_per_step": int(B * sess.in_image_bytes), "d2h_bytes_per_step": int(B * sess.out_bytes),
                      "path": "GraphSession.run_async (C ABI ixb_session_submit / ixb_session_wait_ticket, the "
                              "reference's run_async / RunHandle.wait): pinned host images -> H2D stream -> graph "
                              f"on the compute stream -> D2H stream -> pinned host int8 heads, {depth} batches in "
                              "flight; CUDA events from the first H2D to the last D2H"},
        "roofline": {"bound": "hbm", "kernel": "ixb::conv_kernel (all conv launches of one step)",
                     "achieved": round(achieved_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / hbm_peak, 4), "traffic": traffic,
                     "traffic_source": "profiles/conv_traffic.json: dram__bytes_read.sum + dram__bytes_write.sum "
                                       "of the step's conv launches from one ncu capture (one pass)",
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "algorithmic_bytes_per_step": int(nbytes),
                     "conv_ms_per_step": round(conv_ms, 4),
                     "conv_time_source": "length of the union over the step's conv launches of [inputs ready, "
                                         "last CTA end] (the members of a branch group overlap), traced inside "
                                         "the step's CUDA graph (ixb_session_trace)",
                     "traced_span_ms": round(span_ms, 4),
                     "conv_ms_le_step": bool(conv_ms <= ms / args.steps),
                     "int8_tops": round(int8_tops, 1),
                     "int8_tc_frac": round(int8_tops / (2 * bf16_peak), 4),
                     "int8_tc_peak_note": f"2 x {peak_kind} dense bf16 burst ({bf16_peak} TF/s): int8 runs at twice "
                                          f"the bf16 rate on tcgen05"},
        "gpu_launches": int(launches * args.steps + (launches + 1) * args.steps + launches * args.steps),
        "gpu_launches_note": "device steps (ingress + convs + SPPF per step), then the e2e heads steps and the "
                             "e2e detection steps (+ the decode kernel)",
        "clocks": clocks.summary(),
        "copy_ceiling": ceiling,
        "host_numa_node": numa,
        "per_layer": rows,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    sess.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------- GEMM microbenchmarks
GEMM_SHAPES = [(256, 256, 256), (1024, 1024, 1024), (4096, 4096, 4096), (8192, 8192, 8192),
               (160 * 160 * 64, 16, 144), (160 * 160 * 64, 32, 288), (80 * 80 * 64, 64, 576),
               (80 * 80 * 64, 80, 720), (40 * 40 * 64, 128, 1152), (20 * 20 * 64, 256, 2304)]
W4A8_SHAPES = [(4096, 11008), (11008, 4096)]   # (K, N) of the MLP projections
GEMV_CHAIN = 8                                   # weight images per GEMV chain (8 x 22.5 MB > L2)


def _time_events(fn, iters, warmup, flush=None):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def run_gemm_workloads(args):
    """int8 GEMM + SRS (config: M=N=K sweep and YOLOv8n convs as im2col GEMMs) and W4A8 (MLP
    projections at M=512 prefill and M=1 GEMV): one JSON line, per-shape device times with CUDA
    events, L2 flushed between launches, torch._int_mm (cuBLASLt int8) timed beside the GEMM."""
    import ctypes as C
    import numpy as np
    import torch
    from ignite_xdna_b200 import _lib as L
    lib = L.load()
    hbm, bf16, kind = load_peaks()
    int8_peak = 2 * bf16
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    rows = []
    if args.workload == "i8gemm":
        for M, N, K in GEMM_SHAPES:
            a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
            b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
            bias = torch.randint(-(1 << 20), 1 << 20, (N,), dtype=torch.int32, device="cuda", generator=g)
            out = torch.empty((M, N), dtype=torch.int8, device="cuda")
            fn = lambda: L.check(lib.ixb_i8gemm_srs(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()),  # noqa: E731
                                                    C.c_void_p(bias.data_ptr()), C.c_void_p(out.data_ptr()),
                                                    M, N, K, 8, None))
            ms = _time_events(fn, args.steps, args.warmup, flush)
            bt = b.t()
            ms_lib = _time_events(lambda: torch._int_mm(a, bt), args.steps, args.warmup, flush)
            tops = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            rows.append({"M": M, "N": N, "K": K, "ms": round(ms, 4), "tops": round(tops, 1),
                         "tc_frac": round(tops / int8_peak, 4),
                         "hbm_gbs": round((M * K + N * K + M * N) / (ms * 1e-3) / 1e9, 1),
                         "cublaslt_int_mm_ms": round(ms_lib, 4),
                         "cublaslt_tops": round(2.0 * M * N * K / (ms_lib * 1e-3) / 1e12, 1)})
        head = rows[3]
        metric, unit, value = "int8 GEMM + pow2 SRS TOP/s at M=N=K=8192", "TOP/s", head["tops"]
        roof = {"bound": "tensor", "achieved": head["tops"], "peak": round(int8_peak, 1), "unit": "TFLOP/s",
                "frac": head["tc_frac"], "traffic": None,
                "peak_source": f"2 x {kind} dense bf16 ({bf16} TF/s, MEASURED_PEAKS.json): int8 rate of tcgen05"}
    else:
        rng = np.random.default_rng(0)
        for K, N in W4A8_SHAPES:
            w = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
            wk = ((w[:, 0::2].astype(np.int16) & 0xF) | ((w[:, 1::2].astype(np.int16) & 0xF) << 4)).astype(np.uint8)
            gpos = (5 + rng.integers(0, 4, size=(K // 128, N))).astype(np.int8)
            nbytes = C.c_uint64()
            L.check(lib.ixb_w4a8_image_bytes(K, N, C.byref(nbytes)))
            img = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
            dw, dg = torch.from_numpy(wk).cuda(), torch.from_numpy(gpos).cuda()
            L.check(lib.ixb_w4a8_prepare(C.c_void_p(dw.data_ptr()), C.c_void_p(dg.data_ptr()), K, N,
                                         C.c_void_p(img.data_ptr()), None))
            shift = torch.full((N,), 10, dtype=torch.int32, device="cuda")
            for M in (512, 1):
                a = torch.randn((M, K), device="cuda", generator=g).mul_(24).round_().clamp_(-127, 127).to(torch.int8)
                out = torch.empty((M, N), dtype=torch.int8, device="cuda")
                if M == 1:
                    fn = lambda: L.check(lib.ixb_w4a8_gemv(C.c_void_p(a.data_ptr()), C.c_void_p(img.data_ptr()),  # noqa: E731
                                                           C.c_void_p(shift.data_ptr()), C.c_void_p(out.data_ptr()),
                                                           N, K, None))
                else:
                    fn = lambda: L.check(lib.ixb_w4a8_gemm(C.c_void_p(a.data_ptr()), C.c_void_p(img.data_ptr()),  # noqa: E731
                                                           C.c_void_p(shift.data_ptr()), C.c_void_p(out.data_ptr()),
                                                           M, N, K, None))
                ms = _time_events(fn, args.steps, args.warmup, flush)
                wbytes = K * N // 2 + N * (K // 128)
                rows.append({"M": M, "N": N, "K": K, "ms": round(ms, 4),
                             "tops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 2),
                             "hbm_gbs": round((wbytes + M * K + M * N) / (ms * 1e-3) / 1e9, 1),
                             "kernel": "ixb_w4a8_gemv (streaming 16-byte loads, warp per column)" if M == 1
                             else "ixb_w4a8_gemm (tcgen05, int4 unpack warps)"})
        # the GEMV as a decode step runs it: back to back over distinct weight images whose total
        # (8 x 22.5 MB) exceeds the L2, so every launch streams its weights from DRAM with no flush
        chain = []
        for K, N in W4A8_SHAPES:
            nbytes = C.c_uint64()
            L.check(lib.ixb_w4a8_image_bytes(K, N, C.byref(nbytes)))
            imgs = [torch.randint(0, 256, (nbytes.value,), dtype=torch.uint8, device="cuda", generator=g)
                    for _ in range(GEMV_CHAIN)]
            for im in imgs:  # exponents 4 (d = 0): any bytes are a valid packed operand
                im[N * K // 2:].fill_(4)
            shift = torch.full((N,), 10, dtype=torch.int32, device="cuda")
            a1 = torch.randint(-127, 128, (1, K), dtype=torch.int8, device="cuda", generator=g)
            o1 = torch.empty((GEMV_CHAIN, N), dtype=torch.int8, device="cuda")

            def chain_step(st=None):
                for j, im in enumerate(imgs):
                    L.check(lib.ixb_w4a8_gemv(C.c_void_p(a1.data_ptr()), C.c_void_p(im.data_ptr()),
                                              C.c_void_p(shift.data_ptr()), C.c_void_p(o1[j].data_ptr()), N, K, st))
            ms_eager = _time_events(chain_step, args.steps, args.warmup) / GEMV_CHAIN
            eager_out = o1.clone()
            # a decode step runs its layers from a CUDA graph: the same launches, captured once
            # (programmatic dependent launch edges included), replayed without host launch costs
            side = torch.cuda.Stream()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                chain_step(side.cuda_stream)
                side.synchronize()
                with torch.cuda.graph(graph, stream=side):
                    chain_step(side.cuda_stream)
            o1.zero_()
            ms = _time_events(graph.replay, args.steps, args.warmup) / GEMV_CHAIN
            wbytes = K * N // 2 + N * (K // 128)
            chain.append({"M": 1, "N": N, "K": K, "us_per_gemv": round(ms * 1e3, 2),
                          "hbm_gbs": round((wbytes + K + N) / (ms * 1e-3) / 1e9, 1),
                          "us_per_gemv_host_launched": round(ms_eager * 1e3, 2),
                          "hbm_gbs_host_launched": round((wbytes + K + N) / (ms_eager * 1e-3) / 1e9, 1),
                          "graph_equals_host_launched": bool(torch.equal(o1, eager_out)),
                          "weights_total_mb": round(GEMV_CHAIN * wbytes / 2**20, 1)})
            del graph, imgs
        metric = "W4A8 GEMV weight-stream GB/s (K=4096,N=11008 and K=11008,N=4096)"
        unit = "GB/s"
        value = round(statistics.mean(r["hbm_gbs"] for r in chain), 1)
        roof = {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s", "frac": round(value / hbm, 4),
                "traffic": None, "peak_source": f"{kind} hbm_gbs (MEASURED_PEAKS.json)",
                "value_source": f"a CUDA graph of {GEMV_CHAIN} GEMVs back to back over {GEMV_CHAIN} weight images "
                                "(more bytes than the L2; host-launched chain beside it in gemv_chain); "
                                "the per-shape rows time single launches after a 256 MiB L2 flush"}
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 x int8 -> int32" if args.workload == "i8gemm" else "int8 x int4 -> int32",
            "data": "synthetic (seeded uniform operands)", "config": {"workload": args.workload,
                                                                        "l2": "256 MiB written between launches"},
            "roofline": roof, "shapes": rows, "gpu_launches": len(rows) * args.steps}
    if args.workload == "w4a8":
        line["gemv_chain"] = chain
        line["config"]["l2"] = ("rows: 256 MiB written between launches; value: a chain of GEMVs over "
                                f"{GEMV_CHAIN} distinct weight images, more bytes than the L2")
        line["gpu_launches"] += 2 * len(W4A8_SHAPES) * args.steps * GEMV_CHAIN
    print(json.dumps(line), flush=True)
    return 0


def run_decode_workload(args):
    """The detection stage alone: decode + NMS (ixb_decode_yolo) of `batch` images' int8 heads, the
    network's egress for seeded uniform images, resident on the device (77 MB at batch 64, in L2
    between launches), at two threshold settings. One JSON line: ms per batch and images/s, with a
    SHA-256 of every image's detections so builds can be compared."""
    import ctypes as C
    import hashlib
    import numpy as np
    import torch
    from ignite_xdna_b200 import InferenceSession, random_images
    from ignite_xdna_b200 import _lib as L
    from ignite_xdna_b200.decode import GpuDecoder
    B = args.batch
    sess = InferenceSession.from_spec(args.model, imgsz=args.imgsz, max_batch=B)
    sess.stage_input(random_images(B, args.imgsz, seed=100))
    lib = sess.lib
    L.check(lib.ixb_session_run(sess._h, None, B, None, L.IN_DEVICE | L.OUT_DEVICE | L.ASYNC))
    L.check(lib.ixb_session_wait(sess._h, 60000))
    eg = sess.arena[sess.plan.egress_offset:sess.plan.egress_offset + B * sess.out_bytes]
    rows = []
    for conf, iou in ((0.25, 0.5), (0.5, 0.7)):
        dec = GpuDecoder(sess.layout, args.imgsz, sess.device, conf=conf, iou=iou)
        cap = dec.total_anchors
        lb = torch.zeros((B, 3), dtype=torch.float32, device=sess.device)
        lb[:, 2] = 1.0
        boxes = torch.empty((B, cap, 4), dtype=torch.float32, device=sess.device)
        scores = torch.empty((B, cap), dtype=torch.float32, device=sess.device)
        classes = torch.empty((B, cap), dtype=torch.int32, device=sess.device)
        counts = torch.empty(B, dtype=torch.int32, device=sess.device)
        fn = lambda: L.check(lib.ixb_decode_yolo(  # noqa: E731
            C.byref(dec.desc), C.c_void_p(eg.data_ptr()), B, dec.layout.image_bytes, C.c_void_p(lb.data_ptr()), cap,
            C.c_void_p(boxes.data_ptr()), C.c_void_p(scores.data_ptr()), C.c_void_p(classes.data_ptr()),
            C.c_void_p(counts.data_ptr()), None))
        ms = _time_events(fn, args.steps, args.warmup)
        n = counts.cpu().numpy()
        h = hashlib.sha256()
        for i in range(B):
            k = int(n[i])
            h.update(np.int32(k).tobytes())
            if k > 0:
                for t in (boxes[i, :k], scores[i, :k], classes[i, :k]):
                    h.update(t.cpu().numpy().tobytes())
        rows.append({"conf": conf, "iou": iou, "ms_per_batch": round(ms, 4), "images_s": round(B / (ms * 1e-3), 1),
                     "kept_mean": round(float(n.mean()), 1), "candidates_per_image": cap,
                     "detections_sha256": h.hexdigest()[:16]})
    sess.close()
    line = {"metric": "YOLOv8 detect decode + NMS images/s (GPU, heads resident)", "value": rows[0]["images_s"],
            "unit": "images/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 heads -> float32 (reference order)",
            "data": "synthetic (the network's heads for seeded uniform images)",
            "config": {"workload": f"decode {args.model} {args.imgsz} batch {B}",
                       "l2": "the 77 MB of heads stay in L2 between launches (the decode reads each byte once)"},
            "rows": rows, "gpu_launches": 2 * args.steps}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ixb", choices=["ixb", "reference"])
    ap.add_argument("--model", default="yolov8n", choices=["yolov8n", "yolov8s", "yolov8m"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--depth", type=int, default=4,
                    help="batches in flight in the e2e legs (the session's staging/egress slots, 1..4)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--workload", default="yolo", choices=["yolo", "i8gemm", "w4a8", "decode"],
                    help="yolo: the whole-network benchmark; i8gemm / w4a8 / decode: the kernel microbenchmarks")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "decode":
        return run_decode_workload(args)
    if args.workload != "yolo":
        return run_gemm_workloads(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
