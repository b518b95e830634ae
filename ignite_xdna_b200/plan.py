"""Lower a layer IR to the device plan: storage, packed weights and per-layer descriptors.

HBM layout (one arena per GPU, sized for ``max_batch`` images):

* image staging, uint8 [B][3][H][W], and the pixel -> int8 input table;
* the stem input, int8 [B][H+2][W+4][8] (3 channels + 5 zero bytes per pixel, one zero halo
  column on the left and three on the right, so 16-byte pixel pairs cover every stem window);
* activation buffers: one plane per 16-channel chunk, int8 [B][h+2][w+2][16] with a one-pixel
  zero halo per image and zero guard pixels before and after the plane (a window copy may
  reach past the first and last image). Tensors read together as one concat (a C2f's cv1/m
  outputs, SPPF's cv1 and pools, the PAN concats at one resolution) share a buffer as
  consecutive chunk planes, so the concat is free and every producer writes whole planes of
  its own. Stored values are t = q - 128;
* the egress, int8 [B][egress bytes]: the six heads as NCHW, back to back in head order, the
  head convs write it directly (read_heads' int8 NCHW egress, graph_session.py:903-930);
* constants: weights packed per (n-tile, K-block) in the UMMA core-matrix layout, int32
  biases, the int8 activation tables.

The K order is the kernel's: ``_lib.conv_schedule`` returns the schedule the library builds for a
conv (which input chunks each K-block loads and which (tap, chunk) pairs each MMA multiplies),
and ``pack_weights`` lays the weights out in exactly that order.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import _lib as L
from .graph import ConvLayer, GraphIR, PoolLayer, Segment

ALIGN = 256
TILE_M = 128


def _align(x: int, a: int = ALIGN) -> int:
    return (x + a - 1) // a * a


@dataclass
class Store:
    """Where one tensor lives: chunk plane 0's padded pixel 0, plane stride, first chunk."""
    offset: int
    plane_stride: int
    chunk_offset: int
    channels: int
    height: int
    width: int
    guard: int = 0


def plane_guard(width: int) -> int:
    """Zero pixels around a plane: a window copy reaches up to a 2048-row tile plus one padded
    row and pixel past the last image, and one padded row and pixel before the first."""
    return 2048 + 2 * (width + 3) + 64


def plane_stride(batch: int, height: int, width: int, guard: int) -> int:
    """Bytes per chunk plane: the images plus both guards, rounded up to whole images so a tensor
    map can address chunk c, image n as image c * (stride / image bytes) + n."""
    img = (height + 2) * (width + 2) * 16
    return -(-(batch * img + 2 * guard * 16) // img) * img


@dataclass
class ConvPlan:
    layer: ConvLayer
    mode: int
    n_tile: int
    cp: int
    w_packed: np.ndarray
    desc: Optional[object] = None
    s2d: bool = False  # a stride-2 3x3 run as a 2x2 WINDOW conv over its input's space-to-depth view
    stem_s2d: bool = False  # the stem as a 2x2 WINDOW conv over the image's space-to-depth view


@dataclass
class DevicePlan:
    ir: GraphIR
    max_batch: int
    img_h: int
    img_w: int
    arena_bytes: int
    images_offset: int
    input_lut_offset: int
    input_store: Store
    egress_offset: int
    egress_image_bytes: int
    head_offsets: Dict[str, int]
    stores: Dict[str, Store]
    convs: List[ConvPlan]
    pools: List[Tuple[PoolLayer, object]]
    ops: List[Tuple[int, int]]
    const_offset: int
    const_blob: np.ndarray
    extra_images_offsets: Tuple[int, ...] = ()
    extra_egress_offsets: Tuple[int, ...] = ()
    upsampled_stores: Dict[str, Store] = field(default_factory=dict)  # 2x2 copies (upsampled_copies)
    s2d_stores: Dict[str, Store] = field(default_factory=dict)        # space-to-depth views (s2d_convs)
    s2d_only: frozenset = frozenset()  # tensors stored only as their space-to-depth view
    input_s2d_store: Optional[Store] = None  # the image's space-to-depth view, when the stem reads it
    c_plan: object = None
    keep: list = field(default_factory=list)


def input_lut_t(scale: float) -> np.ndarray:
    """int8 table pixel -> t = clip(round(p/255/s) + 128, 0, 255) - 128 (graph_session.py:144-149)."""
    pixel = np.arange(256, dtype=np.float64) / 255.0
    q = np.clip(np.round(pixel / scale).astype(np.int64) + 128, 0, 255)
    return (q - 128).astype(np.int8)


def upsampled_copies(ir: GraphIR) -> set:
    """Conv outputs that a later conv reads nearest-2x upsampled (the top-down path's Resize into
    Concat). Their producing conv also writes a 2x2-replicated copy at twice the resolution, so the
    consumer reads a plain tensor through bulk copies (WINDOW) instead of gathering 16-byte rows
    (GATHER). On YOLOv8n at batch 64 that took the two concat 1x1 convs from 48 and 26 us to 24 and
    17 us, while their producers went from 12 to 21 and 18 us (four times the output writes):
    1.300 -> 1.282 ms per step.
    IXB_UP2=0 keeps the gathers (the GATHER kernel stays covered by the tests that way)."""
    if os.environ.get("IXB_UP2", "1") == "0":
        return set()
    produced = {layer.output for layer in ir.conv_layers()}
    return {s.tensor for layer in ir.conv_layers() for s in layer.inputs if s.up2 and s.tensor in produced}


def s2d_convs(ir: GraphIR) -> set:
    """Stride-2 3x3 convs run as stride-1 2x2 WINDOW convs over the space-to-depth view of their
    input (four phase planes (row parity, column parity) at half resolution, written by the
    input's producing conv), so their A operand comes in bulk copies instead of TMA im2col loads
    of one 16-byte pixel per row. Needs a conv-produced input of whole chunks and even size;
    IXB_S2D=0 keeps the im2col loads (the IM2COL kernel stays covered by the tests that way)."""
    if os.environ.get("IXB_S2D", "1") == "0":
        return set()
    produced = {layer.output for layer in ir.conv_layers()}
    out = set()
    for layer in ir.conv_layers():
        if layer.k != 3 or layer.stride != 2 or len(layer.inputs) != 1:
            continue
        s = layer.inputs[0]
        t = ir.tensors[s.tensor]
        if (s.tensor in produced and not s.up2 and s.block_offset == 0 and s.blocks * 8 == t.channels
                and t.channels % 16 == 0 and t.height % 2 == 0 and t.width % 2 == 0
                and 9 * (t.channels // 16) <= 300):   # <= 150 MMAs in the kernel's op table
            out.add(layer.name)
    return out


def _s2d_k(d: int, r: int) -> Optional[int]:
    """The 3x3 tap (ky or kx) that a 2x2 space-to-depth tap d in {-1, 0} reads in phase r, or None:
    input row 2y + ky - 1 is phase 1 one row back for ky = 0, phase 0 for 1, phase 1 for 2."""
    if d == -1:
        return 0 if r == 1 else None
    return 1 if r == 0 else 2


def stem_s2d_piece(w: np.ndarray):
    """(chunk 0, tap) -> [cout, 16] weights of the stem over the image's space-to-depth view: byte
    ph * 3 + c of a pixel is channel c of phase ph = 2 ry + rx; bytes 12..15 are zero."""
    def piece(chunk, tap):
        out = np.zeros((w.shape[0], 16), dtype=np.int8)
        for ph in range(4):
            ry, rx = divmod(ph, 2)
            ky, kx = _s2d_k(tap // 2 - 1, ry), _s2d_k(tap % 2 - 1, rx)
            if ky is not None and kx is not None:
                out[:, 3 * ph:3 * ph + 3] = w[:, :, ky, kx]
        return out
    return piece


def s2d_weight_piece(w: np.ndarray, chunks: int):
    """(chunk, tap) -> [cout, 16] weights of a 3x3 stride-2 conv run over the space-to-depth view:
    chunk c is phase (ry, rx) = divmod(c // chunks, 2) of input chunk c % chunks, tap t of the 2x2 is
    (dy, dx) = (t // 2 - 1, t % 2 - 1). Input row 2y + ky - 1 is phase 1, one row back, for ky = 0,
    phase 0 for ky = 1 and phase 1 for ky = 2 (columns alike); pairs the 3x3 never reads are zero."""
    def k_of(d, r):
        if d == -1:
            return 0 if r == 1 else None
        return 1 if r == 0 else 2

    def piece(chunk, tap):
        ry, rx = divmod(chunk // chunks, 2)
        c = chunk % chunks
        ky, kx = k_of(tap // 2 - 1, ry), k_of(tap % 2 - 1, rx)
        if ky is None or kx is None:
            return np.zeros((w.shape[0], 16), dtype=np.int8)
        return np.ascontiguousarray(w[:, 16 * c:16 * c + 16, ky, kx])
    return piece


def conv_mode(layer: ConvLayer, ir: GraphIR, upsampled: frozenset = frozenset()) -> int:
    if layer.inputs[0].tensor == ir.input:
        return L.MODE_STEM
    if any(s.up2 and s.tensor not in upsampled for s in layer.inputs):
        return L.MODE_GATHER
    if layer.stride == 1:
        return L.MODE_WINDOW
    if layer.k == 3 and layer.stride == 2 and len({s.tensor for s in layer.inputs}) == 1:
        return L.MODE_IM2COL
    raise ValueError(f"{layer.name}: no conv mode for k={layer.k} stride={layer.stride}")


def pad16(c: int) -> int:
    """Channels as stored: whole 16-channel chunks (a tensor of 51 or 1 channels keeps zero channels
    up to its last chunk; its producer has zero weights and bias there, its consumers zero weights)."""
    return (c + 15) // 16 * 16


def choose_n_tile(cout: int) -> int:
    if cout <= 256:
        return cout
    for n in range(256, 15, -16):
        if cout % n == 0:
            return n
    raise ValueError(f"no n-tile for {cout} output channels")


def choose_cp(mode: int, k: int, cin: int) -> int:
    if mode == L.MODE_STEM:
        return 2
    pairs = (cin + 31) // 32
    if mode == L.MODE_WINDOW and k == 2:
        # the 2x2 space-to-depth form: 9 of its 16 (phase, tap) pairs carry weights, so a K-block of
        # one chunk pair may hold a single MMA; two pairs per K-block measured 15-25 % faster on the
        # 40x40 and 20x20 layers (>= 256 view channels) and slower on the 160x160 one
        return 2 if cin >= 256 else 1
    if (mode == L.MODE_WINDOW and k == 3) or mode == L.MODE_IM2COL:
        return 1    # 3x3: a K-block already carries the MMAs of 9 (window) or 3 (im2col) taps per pair
    return 4 if pairs >= 4 else (2 if pairs >= 2 else 1)


def _core_layout(b: np.ndarray) -> np.ndarray:
    """[n, 32] K-major bytes -> UMMA no-swizzle core matrices [n/8][2][8][16]."""
    n = b.shape[0]
    return b.reshape(n // 8, 8, 2, 16).transpose(0, 2, 1, 3).reshape(-1)


def pack_weights(layer: ConvLayer, mode: int, n_tile: int, schedule,
                 cin_map: Optional[np.ndarray] = None, s2d: bool = False, stem_s2d: bool = False) -> np.ndarray:
    """Weights of every n-tile as the schedule's MMAs' [n_tile][32] K-slices, each in the UMMA
    core-matrix layout; a slice's two 16-byte K-halves are the (chunk, tap) of the MMA's halves.
    ``cin_map`` places input channel i at stored channel cin_map[i] (inputs padded to whole chunks);
    the stored channels it does not name get zero weights."""
    w = layer.weights.astype(np.int8)       # [cout][cin][k][k]
    if w.shape[0] % n_tile:                 # output channels padded to whole chunks: zero weights
        w = np.concatenate([w, np.zeros((pad16(w.shape[0]) - w.shape[0],) + w.shape[1:], np.int8)])
    cout, cin, k, _ = w.shape
    nchunks = (cin + 15) // 16
    if stem_s2d:
        piece = stem_s2d_piece(w)
    elif mode == L.MODE_STEM:
        # tap 2*ky + p is the 16-byte pixel pair p of image row ky: image pixel 2x + 2p + j (j = 0, 1)
        # at kx = 2p + j, bytes 8*j + ci; kx = 3 and channels 3..7 are zero
        stem = np.zeros((6, cout, 16), dtype=np.int8)
        for ky in range(3):
            for kx in range(3):
                pr, j = divmod(kx, 2)
                for ci in range(3):
                    stem[2 * ky + pr, :, 8 * j + ci] = w[:, ci, ky, kx]

        def piece(chunk, tap):
            return stem[tap]
    elif s2d:
        piece = s2d_weight_piece(w, nchunks)
    else:
        if cin_map is None:
            cin_map = np.arange(cin)
        wp = np.zeros((cout, (int(cin_map[-1]) + 16) // 16 * 16, k * k), dtype=np.int8)
        wp[:, cin_map, :] = w.reshape(cout, cin, k * k)

        def piece(chunk, tap):
            return wp[:, 16 * chunk:16 * chunk + 16, tap]
    zero = np.zeros((cout, 16), dtype=np.int8)
    out = []
    for nt in range(cout // n_tile):
        sl = slice(nt * n_tile, (nt + 1) * n_tile)
        for blk in schedule:
            for (_, c0, t0), second in blk["ops"]:
                h0 = piece(c0, t0)
                h1 = piece(second[1], second[2]) if second is not None else zero
                out.append(_core_layout(np.ascontiguousarray(np.concatenate([h0[sl], h1[sl]], axis=1))))
    return np.concatenate(out).view(np.uint8)


def _storage_groups(ir: GraphIR, heads: set) -> List[List[str]]:
    """Tensors read together as a concat at one resolution, in channel order."""
    grouped: Dict[str, int] = {}
    groups: List[List[str]] = []
    for layer in ir.conv_layers():
        run: List[str] = []

        def flush():
            if len(run) >= 2 and not any(t in grouped for t in run):
                for t in run:
                    grouped[t] = len(groups)
                groups.append(list(run))
            run.clear()

        for s in layer.inputs:
            t = ir.tensors[s.tensor]
            whole = s.block_offset == 0 and s.blocks * 8 == t.channels
            if s.up2 or not whole or s.tensor == ir.input or s.tensor in run:
                flush()
                continue
            run.append(s.tensor)
        flush()
    for name in ir.tensors:
        if name not in grouped and name != ir.input and name not in heads:
            groups.append([name])
    return groups


def _cin_map(ir: GraphIR, layer: ConvLayer) -> np.ndarray:
    """Stored channel of each of the layer's input channels across its (padded) segments."""
    parts, base = [], 0
    for s in layer.inputs:
        t = ir.tensors[s.tensor]
        parts.append(base + np.arange(min(s.blocks * 8, t.channels - s.block_offset * 8)))
        base += _seg_channels(ir, s)
    m = np.concatenate(parts)
    if m.size != layer.cin:
        raise ValueError(f"{layer.name}: segments carry {m.size} channels, weights {layer.cin}")
    return m


def _seg_channels(ir: GraphIR, s: Segment) -> int:
    """Channels a segment view reads as stored: whole chunks; a view that ends inside a chunk must
    end at its tensor's last channel (the stored zero channels then complete the chunk)."""
    if s.tensor == ir.input:
        return 3
    t = ir.tensors[s.tensor]
    if s.block_offset % 2:
        raise ValueError(f"{s.tensor}: channel view not aligned to 16-channel chunks")
    real = min(s.blocks * 8, t.channels - s.block_offset * 8)
    if real % 16:
        if s.block_offset * 8 + real != t.channels:
            raise ValueError(f"{s.tensor}: channel view ends inside a 16-channel chunk")
        real = pad16(real)
    return real


def branch_schedule(ir: GraphIR, ops: List[Tuple[int, int]], convs, pools) -> List[Tuple[int, int]]:
    """Reorder ``ops`` into dependency levels (an op's level is one more than its latest input's
    producer) and join each level's convs into branch groups of at most ``MAX_BRANCHES`` with the
    ``OP_WITH_PREV`` flag: every op of a level reads only tensors of earlier levels and no tensor
    is written twice, so a level's convs are independent and may run concurrently. Pools stay
    alone, ahead of their level's convs."""
    def rw(kind, idx):
        if kind == L.OP_CONV:
            layer = convs[idx].layer
            reads = {s.tensor for s in layer.inputs}
            if layer.residual is not None:
                reads.add(layer.residual.tensor)
            return reads, {layer.output}
        chain = pools[idx][0]
        return {chain[0].input.tensor}, {p.output for p in chain}
    producer: Dict[str, int] = {}
    level: List[int] = []
    for i, (kind, idx) in enumerate(ops):
        reads, writes = rw(kind, idx)
        level.append(1 + max((level[producer[t]] for t in reads if t in producer), default=0))
        for t in writes:
            if t in producer:
                raise ValueError(f"tensor {t} written twice")
            producer[t] = i
    out: List[Tuple[int, int]] = []
    for lv in sorted(set(level)):
        members = [i for i in range(len(ops)) if level[i] == lv]
        for i in members:
            if ops[i][0] != L.OP_CONV:
                out.append(ops[i])
        run = 0
        for i in members:
            if ops[i][0] != L.OP_CONV:
                continue
            flag = L.OP_WITH_PREV if 0 < run < L.MAX_BRANCHES else 0
            run = run + 1 if flag else 1
            out.append((ops[i][0] | flag, ops[i][1]))
    return out


def build_plan(ir: GraphIR, max_batch: int, pipeline_depth: int = 3, branches: Optional[bool] = None) -> DevicePlan:
    """Arena layout, packed constants and kernel descriptors for ``ir`` at up to ``max_batch``
    images; ``pipeline_depth`` staging/egress pairs serve the submitted-run ring. With
    ``branches`` (default: on unless IXB_BRANCHES=0) independent convs of one dependency level
    form branch groups that run concurrently on forked streams, the SMs split in proportion to
    each member's measured time alone (the YOLOv8n 640x640 batch-64 step: 1.086 ms against
    1.110 ms in the graph's serial order)."""
    if max_batch < 1:
        raise ValueError("max_batch must be >= 1")
    if not 1 <= pipeline_depth <= 1 + L.MAX_EXTRA_SLOTS:
        raise ValueError(f"pipeline_depth must be in [1, {1 + L.MAX_EXTRA_SLOTS}]")
    timg = ir.tensors[ir.input]
    H, W = timg.height, timg.width
    head_tensor = dict(ir.outputs)
    heads = set(head_tensor.values())
    off = 0

    def alloc(nbytes: int) -> int:
        nonlocal off
        o = off
        off = _align(off + nbytes)
        return o

    images_offset = alloc(max_batch * 3 * H * W)
    extra_images = tuple(alloc(max_batch * 3 * H * W) for _ in range(pipeline_depth - 1))
    input_lut_offset = alloc(256)
    input_store = Store(alloc(max_batch * (H + 2) * (W + 4) * 8), 0, 0, 3, H, W, 0)
    # the stem over the image's space-to-depth view (one 16-byte chunk: 4 phases x 3 channels),
    # fed by bulk copies instead of TMA im2col loads of 16-byte pixel pairs
    input_s2d_store = None
    if os.environ.get("IXB_S2D", "1") != "0" and H % 2 == 0 and W % 4 == 0:
        guard = plane_guard(W // 2)
        plane = plane_stride(max_batch, H // 2, W // 2, guard)
        input_s2d_store = Store(alloc(plane) + guard * 16, plane, 0, 16, H // 2, W // 2, guard)
    stores: Dict[str, Store] = {}
    for grp in _storage_groups(ir, heads):
        infos = [ir.tensors[t] for t in grp]
        for t in infos:
            if t.channels % 16 and len(infos) > 1:
                raise ValueError(f"{t.name}: a concatenated tensor of {t.channels} channels (not whole chunks)")
        h, w = infos[0].height, infos[0].width
        guard = plane_guard(w)
        plane = plane_stride(max_batch, h, w, guard)
        nch = sum(pad16(t.channels) for t in infos) // 16
        base = alloc(nch * plane) + guard * 16
        ch = 0
        for t in infos:
            stores[t.name] = Store(base, plane, ch, pad16(t.channels), h, w, guard)
            ch += pad16(t.channels) // 16
    # the 2x2-replicated copies of upsampled conv outputs (see upsampled_copies)
    upsampled = upsampled_copies(ir)
    stores_up2: Dict[str, Store] = {}
    for name in sorted(upsampled):
        t = ir.tensors[name]
        h, w = 2 * t.height, 2 * t.width
        guard = plane_guard(w)
        plane = plane_stride(max_batch, h, w, guard)
        base = alloc(pad16(t.channels) // 16 * plane) + guard * 16
        stores_up2[name] = Store(base, plane, 0, pad16(t.channels), h, w, guard)
    # the space-to-depth views of the stride-2 convs' inputs (see s2d_convs)
    s2d_layers = s2d_convs(ir)
    s2d_src = {layer.inputs[0].tensor for layer in ir.conv_layers() if layer.name in s2d_layers}
    stores_s2d: Dict[str, Store] = {}
    for name in sorted(s2d_src):
        t = ir.tensors[name]
        h, w = t.height // 2, t.width // 2
        guard = plane_guard(w)
        plane = plane_stride(max_batch, h, w, guard)
        base = alloc(4 * pad16(t.channels) // 16 * plane) + guard * 16
        stores_s2d[name] = Store(base, plane, 0, 4 * pad16(t.channels), h, w, guard)
    # a tensor read by nothing but its space-to-depth consumers is stored only in that view
    readers: Dict[str, List[str]] = {}
    for layer in ir.layers:
        ins = layer.inputs if isinstance(layer, ConvLayer) else [layer.input]
        for s in ins:
            readers.setdefault(s.tensor, []).append(layer.name)
        if isinstance(layer, ConvLayer) and layer.residual is not None:
            readers.setdefault(layer.residual.tensor, []).append(layer.name)
    s2d_only = frozenset(n for n in s2d_src if n not in heads and all(r in s2d_layers for r in readers[n]))
    head_offsets: Dict[str, int] = {}
    eb = 0
    for name, _ in ir.outputs:
        t = ir.tensors[head_tensor[name]]
        head_offsets[name] = eb
        eb += t.channels * t.height * t.width
    egress_image_bytes = eb
    egress_offset = alloc(max_batch * egress_image_bytes)
    extra_egress = tuple(alloc(max_batch * egress_image_bytes) for _ in range(pipeline_depth - 1))

    # constants
    const_parts: List[Tuple[int, np.ndarray]] = []
    coff = 0

    def cput(a: np.ndarray) -> int:
        nonlocal coff
        o = coff
        const_parts.append((o, np.ascontiguousarray(a).view(np.uint8).reshape(-1)))
        coff = _align(coff + a.nbytes)
        return o

    convs: List[ConvPlan] = []
    for layer in ir.conv_layers():
        s2d = layer.name in s2d_layers
        stem_s2d = input_s2d_store is not None and layer.inputs[0].tensor == ir.input
        mode = L.MODE_WINDOW if s2d or stem_s2d else conv_mode(layer, ir, frozenset(upsampled))
        cin_p = 3 if mode == L.MODE_STEM or stem_s2d else sum(_seg_channels(ir, sg) for sg in layer.inputs)
        cout_p = pad16(layer.cout)
        n_tile = choose_n_tile(cout_p)
        k, stride, cin_k = ((2, 1, 4 * cin_p) if s2d else (2, 1, 16) if stem_s2d else
                            (layer.k, layer.stride, cin_p))
        cp = choose_cp(mode, k, cin_k)
        shape = L.ConvDesc()
        shape.mode, shape.k, shape.stride, shape.n_tile, shape.cp = mode, k, stride, n_tile, cp
        shape.s2d_in = 2 if stem_s2d else int(s2d)
        shape.cin, shape.cout = cin_k, cout_p
        shape.nseg = 1
        shape.seg[0].channels = cin_k
        sched = L.conv_schedule(shape)
        wp = pack_weights(layer, mode, n_tile, sched,
                          None if mode == L.MODE_STEM or s2d or stem_s2d else _cin_map(ir, layer),
                          s2d=s2d, stem_s2d=stem_s2d)
        cpl = ConvPlan(layer, mode, n_tile, cp, wp, s2d=s2d, stem_s2d=stem_s2d)
        cpl.schedule = sched
        cpl.w_rel = cput(wp)
        bias = np.zeros(cout_p, dtype=np.int32)
        bias[:layer.cout] = layer.bias_int8_domain().astype(np.int32)
        cpl.bias_rel = cput(bias)
        cpl.lut_rel = cput(layer.lut_t())
        convs.append(cpl)
    ilut_rel = cput(input_lut_t(timg.scale))
    const_offset = alloc(coff)
    blob = np.zeros(coff, dtype=np.uint8)
    for o, a in const_parts:
        blob[o:o + a.size] = a
    arena_bytes = _align(off, 1 << 20)

    def seg_of(s: Segment) -> L.Segment:
        if s.tensor == ir.input:
            st = input_store
            return L.Segment(st.offset, 0, 0, 3, st.height, st.width, 0, 0)
        if s.up2 and s.tensor in stores_up2:
            st = stores_up2[s.tensor]
            return L.Segment(st.offset, st.plane_stride, st.chunk_offset + s.block_offset // 2,
                             _seg_channels(ir, s), st.height, st.width, 0, st.guard)
        st = stores[s.tensor]
        return L.Segment(st.offset, st.plane_stride, st.chunk_offset + s.block_offset // 2, _seg_channels(ir, s),
                         st.height, st.width, int(s.up2), st.guard)

    def whole(name: str) -> L.Segment:
        st = stores[name]
        return L.Segment(st.offset, st.plane_stride, st.chunk_offset, st.channels, st.height, st.width, 0, st.guard)

    plan_convs = []
    index_of = {}
    for i, cpl in enumerate(convs):
        layer = cpl.layer
        t_out = ir.tensors[layer.output]
        src = ir.tensors[layer.inputs[0].tensor]
        up = 2 if layer.inputs[0].up2 else 1
        d = L.ConvDesc()
        d.mode = cpl.mode
        d.k, d.stride = layer.k, layer.stride
        d.in_h, d.in_w = src.height * up, src.width * up
        d.out_h, d.out_w = t_out.height, t_out.width
        d.cin = sum(_seg_channels(ir, sg) for sg in layer.inputs) if cpl.mode != L.MODE_STEM else 3
        d.cout = pad16(layer.cout)
        d.n_tile, d.cp = cpl.n_tile, cpl.cp
        segs = _merge_segments([seg_of(s) for s in layer.inputs])
        if cpl.stem_s2d:
            st = input_s2d_store
            d.k, d.stride, d.s2d_in = 2, 1, 2
            d.in_h, d.in_w = st.height, st.width
            d.cin = 16
            segs = [L.Segment(st.offset, st.plane_stride, 0, 16, st.height, st.width, 0, st.guard)]
        if cpl.s2d:
            st = stores_s2d[layer.inputs[0].tensor]
            d.k, d.stride, d.s2d_in = 2, 1, 1
            d.in_h, d.in_w = st.height, st.width
            d.cin = st.channels
            segs = [L.Segment(st.offset, st.plane_stride, 0, st.channels, st.height, st.width, 0, st.guard)]
        if len(segs) > L.MAX_SEGS:
            raise ValueError(f"{layer.name}: more than {L.MAX_SEGS} input segments")
        d.nseg = len(segs)
        for j, s in enumerate(segs):
            d.seg[j] = s
        d.w_offset = const_offset + cpl.w_rel
        d.w_bytes = cpl.w_packed.size
        d.bias_offset = const_offset + cpl.bias_rel
        d.lut_offset = const_offset + cpl.lut_rel
        d.shift = layer.shift_out
        if layer.residual is not None:
            d.has_residual = 1
            d.residual = seg_of(layer.residual)
            d.res_lsh_main = layer.residual_lsh_main
            d.res_lsh_res = layer.residual_lsh_res if layer.residual_lsh_res is not None else layer.residual_shift
            d.res_shift = layer.residual_shift
        if layer.output in heads:
            name = [n for n, t in ir.outputs if t == layer.output][0]
            d.out_nchw = 1
            d.egress_offset = egress_offset + head_offsets[name]
            d.egress_image_bytes = egress_image_bytes
            d.egress_channels = layer.cout
        else:
            d.out = whole(layer.output)
        second = stores_up2.get(layer.output) or stores_s2d.get(layer.output)
        if second is not None:
            if layer.output in stores_up2 and layer.output in stores_s2d:
                raise ValueError(f"{layer.output}: both an upsampled and a space-to-depth copy")
            d.out2_kind = (L.OUT2_UP2 if layer.output in stores_up2 else
                           L.OUT2_S2D_ONLY if layer.output in s2d_only else L.OUT2_S2D)
            d.out2 = L.Segment(second.offset, second.plane_stride, 0, second.channels, second.height,
                               second.width, 0, second.guard)
        cpl.desc = d
        plan_convs.append(d)
        index_of[layer.name] = i
    pools = []
    ops: List[Tuple[int, int]] = []
    pool_layers = ir.pool_layers()
    done_pools = set()
    for layer in ir.layers:
        if isinstance(layer, ConvLayer):
            ops.append((L.OP_CONV, index_of[layer.name]))
            continue
        if layer.name in done_pools:
            continue
        # SPPF: three chained pools run as one kernel
        chain = [layer]
        while len(chain) < 3:
            nxt = [p for p in pool_layers if p.input.tensor == chain[-1].output]
            if len(nxt) != 1:
                raise ValueError(f"{layer.name}: expected a chain of three 5x5 pools")
            chain.append(nxt[0])
        pd = L.PoolDesc()
        pd.inp = seg_of(layer.input)
        for k, p in enumerate(chain):
            pd.out[k] = whole(p.output)
            done_pools.add(p.name)
        pools.append((chain, pd))
        ops.append((L.OP_POOL, len(pools) - 1))
    if branches is None:
        branches = os.environ.get("IXB_BRANCHES", "1") != "0"
    if branches:
        ops = branch_schedule(ir, ops, convs, pools)
    return DevicePlan(ir=ir, max_batch=max_batch, img_h=H, img_w=W, arena_bytes=arena_bytes,
                      images_offset=images_offset, input_lut_offset=const_offset + ilut_rel,
                      input_store=input_store, egress_offset=egress_offset, egress_image_bytes=egress_image_bytes,
                      head_offsets=head_offsets, stores=stores, convs=convs, pools=pools, ops=ops,
                      const_offset=const_offset, const_blob=blob, extra_images_offsets=extra_images,
                      extra_egress_offsets=extra_egress, upsampled_stores=stores_up2, s2d_stores=stores_s2d,
                      s2d_only=s2d_only, input_s2d_store=input_s2d_store)


def _merge_segments(segs: List[L.Segment]) -> List[L.Segment]:
    """Adjacent views of one buffer (same planes, consecutive chunks) become one view."""
    out: List[L.Segment] = []
    for s in segs:
        if out:
            p = out[-1]
            if (p.offset == s.offset and p.plane_stride == s.plane_stride and not p.up2 and not s.up2
                    and p.chunk_offset + p.channels // 16 == s.chunk_offset):
                p.channels += s.channels
                continue
        out.append(L.Segment(s.offset, s.plane_stride, s.chunk_offset, s.channels, s.height, s.width, s.up2,
                             s.guard))
    return out


def c_plan(dp: DevicePlan) -> L.Plan:
    """The ixb_plan struct (arrays kept alive on the DevicePlan)."""
    convs = (L.ConvDesc * len(dp.convs))(*[c.desc for c in dp.convs])
    pools = (L.PoolDesc * max(1, len(dp.pools)))(*[p for _, p in dp.pools])
    ops = (L.Op * len(dp.ops))(*[L.Op(k, i) for k, i in dp.ops])
    p = L.Plan()
    p.api_version = L.API_VERSION
    p.max_batch = dp.max_batch
    p.img_h, p.img_w = dp.img_h, dp.img_w
    p.n_convs, p.n_pools, p.n_ops = len(dp.convs), len(dp.pools), len(dp.ops)
    p.convs = convs
    p.pools = pools
    p.ops = ops
    p.images_offset = dp.images_offset
    p.input_lut_offset = dp.input_lut_offset
    s = dp.input_store
    p.input = L.Segment(s.offset, 0, 0, 3, s.height, s.width, 0, 0)
    if dp.input_s2d_store is not None:
        v = dp.input_s2d_store
        p.input_s2d = 1
        p.input_s2d_view = L.Segment(v.offset, v.plane_stride, 0, 16, v.height, v.width, 0, v.guard)
    p.egress_offset = dp.egress_offset
    p.egress_image_bytes = dp.egress_image_bytes
    p.arena_bytes = dp.arena_bytes
    p.extra_slots = len(dp.extra_images_offsets)
    for i, (a, b) in enumerate(zip(dp.extra_images_offsets, dp.extra_egress_offsets)):
        p.extra_images_offset[i] = a
        p.extra_egress_offset[i] = b
    dp.keep = [convs, pools, ops]
    dp.c_plan = p
    return p
