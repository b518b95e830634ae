"""CPU oracle for the XINT8 YOLOv8 path: test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use this
module, and only as the checker or as the timed CPU baseline; the engine never imports it.

It restates, in numpy, the reference's integer reference of the quantized graph
(``src/ignite_xdna/compiler/graph_reference.py``) and the arithmetic it calls from
``src/ignite_xdna/compiler/engine_emulator.py``. It works in the reference's own domain:
uint8 activations with zero point 128, the folded accumulator bias ``bias_acc``, a
float64 tensordot per tap (exact while |acc| < 2^53), then RNE shift, uint8 saturation,
the activation table, and the residual rule. Results are uint8 [C][H][W] per tensor.

Parity is pinned by ``tests/golden/`` fixtures made by running the reference's own
``run_direct`` on the same graphs and inputs (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

from typing import Dict, Iterable, List, Optional

import numpy as np

ZP = 128


def rne_shift(x, s: int) -> np.ndarray:
    """Shift right by s rounding half to even; s <= 0 shifts left (engine_emulator.py:149-158)."""
    x = np.asarray(x, dtype=np.int64)
    if s <= 0:
        return x << (-s)
    q = x >> s
    rem = x - (q << s)
    half = np.int64(1) << (s - 1)
    return q + ((rem > half) | ((rem == half) & ((q & 1) == 1))).astype(np.int64)


def sat_u8(x) -> np.ndarray:
    """engine_emulator.py:161-162."""
    return np.clip(np.asarray(x, dtype=np.int64), 0, 255).astype(np.uint8)


def sat_i16(x) -> np.ndarray:
    """engine_emulator.py:165-166."""
    return np.clip(np.asarray(x, dtype=np.int64), -32768, 32767)


def residual_combine(qm, qr, rsh: int, lsh_m: int = 0, lsh_r: Optional[int] = None) -> np.ndarray:
    """sat_u8(sat16(rne((tm << lsh_m) + (tr << lsh_r), rsh)) + 128) (engine_emulator.py:195-204)."""
    lsh_r = rsh if lsh_r is None else lsh_r
    tm = np.asarray(qm).astype(np.int64) - ZP
    tr = np.asarray(qr).astype(np.int64) - ZP
    return sat_u8(sat_i16(rne_shift((tm << lsh_m) + (tr << lsh_r), rsh)) + ZP)


def input_lut(input_scale: float, input_zero_point: int = ZP) -> np.ndarray:
    """uint8 pixel -> uint8 model input q = clip(round(p/255/s) + zp) (graph_session.py:144-149)."""
    pixel = np.arange(256, dtype=np.float64) / 255.0
    return np.clip(np.round(pixel / input_scale).astype(np.int64) + input_zero_point, 0, 255).astype(np.uint8)


def quantize_image(pixels_chw: np.ndarray, input_scale: float) -> np.ndarray:
    """uint8 pixels [3][H][W] -> uint8 model input (graph_reference.py:20-24 on p/255)."""
    return input_lut(input_scale)[np.asarray(pixels_chw, dtype=np.uint8)]


def gather_input(tensors: Dict[str, np.ndarray], segments, height: int, width: int) -> np.ndarray:
    """Concatenate channel-block views, nearest-2x where flagged (graph_reference.py:27-37)."""
    parts = []
    for s in segments:
        chans = tensors[s.tensor][s.block_offset * 8:(s.block_offset + s.blocks) * 8]
        if s.up2:
            chans = np.repeat(np.repeat(chans, 2, axis=1), 2, axis=2)
        if chans.shape[1:] != (height, width):
            raise ValueError(f"segment {s.tensor} is {chans.shape[1:]}, expected {(height, width)}")
        parts.append(chans)
    return np.concatenate(parts, axis=0)


def conv_accumulate(layer, x: np.ndarray, folded: bool = True) -> np.ndarray:
    """int64 accumulator Σ w·q + bias_acc over the ZP-padded input (graph_reference.py:40-55).

    folded=False gives the same sum in the signed domain t = q - 128 without the zero-point terms:
    Σ w·t + (bias_q << e)."""
    cin, h, w = x.shape
    k, s, p = layer.k, layer.stride, layer.pad
    xp = np.full((cin, h + 2 * p, w + 2 * p), ZP, dtype=np.uint8)
    xp[:, p:p + h, p:p + w] = x
    ho = (h + 2 * p - k) // s + 1
    wo = (w + 2 * p - k) // s + 1
    wts = layer.weights.astype(np.float64)
    acc = np.zeros((wts.shape[0], ho, wo), dtype=np.float64)
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, ky:ky + s * ho:s, kx:kx + s * wo:s].astype(np.float64)
            acc += np.tensordot(wts[:, :, ky, kx], patch, axes=([1], [0]))
    if not folded:
        wsum = layer.weights.astype(np.int64).sum(axis=(1, 2, 3))
        return acc.astype(np.int64) - ZP * wsum[:, None, None] + layer.bias_int8_domain()[:, None, None]
    return acc.astype(np.int64) + layer.bias_acc()[:, None, None]


def conv_direct(layer, x: np.ndarray) -> np.ndarray:
    """uint8 [Cin][H][W] -> uint8 [Cout][Ho][Wo]: SRS, saturate, activation table (graph_reference.py:56-61).

    A negative SRS shift (a layer whose output scale is finer than its input times weight scale)
    cannot be expressed through the reference's folded bias, whose ``128 << shift`` term
    (graph_ir.py:126-134) raises for it; there the oracle applies rne_shift's left-shift rule
    (engine_emulator.py:149-158) to the signed-domain sum and adds the zero point after the
    shift, which for every shift >= 0 is the folded rule exactly."""
    if layer.shift_out < 0:
        q = sat_u8(rne_shift(conv_accumulate(layer, x, folded=False), layer.shift_out) + ZP)
        return layer.sigmoid.table[q] if layer.sigmoid is not None else q
    q = sat_u8(rne_shift(conv_accumulate(layer, x), layer.shift_out))
    if layer.sigmoid is not None:
        q = layer.sigmoid.table[q]
    return q


def maxpool5_direct(x: np.ndarray) -> np.ndarray:
    """5x5 stride-1 max with uint8 0 padding (graph_reference.py:64-72)."""
    c, h, w = x.shape
    xp = np.zeros((c, h + 4, w + 4), dtype=np.uint8)
    xp[:, 2:2 + h, 2:2 + w] = x
    out = np.zeros_like(x)
    for dy in range(5):
        for dx in range(5):
            out = np.maximum(out, xp[:, dy:dy + h, dx:dx + w])
    return out


def run_direct(ir, input_q: np.ndarray, stop_after: Optional[int] = None) -> Dict[str, np.ndarray]:
    """Evaluate the graph on one uint8 image; {tensor name: uint8 [C][H][W]} (graph_reference.py:119-169)."""
    tensors: Dict[str, np.ndarray] = {ir.input: input_q}
    for L in ir.layers:
        if stop_after is not None and L.index > stop_after:
            break
        t = ir.tensors[L.output]
        if hasattr(L, "weights"):
            src = ir.tensors[L.inputs[0].tensor]
            up = 2 if L.inputs[0].up2 else 1
            y = conv_direct(L, gather_input(tensors, L.inputs, src.height * up, src.width * up))
            if L.residual is not None:
                r = gather_input(tensors, [L.residual], t.height, t.width)
                y = residual_combine(y, r, L.residual_shift, L.residual_lsh_main, L.residual_lsh_res)
            tensors[L.output] = y
        else:
            tensors[L.output] = maxpool5_direct(gather_input(tensors, [L.input], t.height, t.width))
    return tensors


def run_image(ir, pixels_chw: np.ndarray) -> Dict[str, np.ndarray]:
    """uint8 pixels [3][H][W] -> every tensor of the graph (uint8, zero point 128)."""
    return run_direct(ir, quantize_image(pixels_chw, ir.tensors[ir.input].scale))


def heads_int8(ir, tensors: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """The six heads as int8 NCHW (q ^ 0x80, zero point 0), as read_heads presents them (graph_session.py:903-930)."""
    return {name: (tensors[t].astype(np.int16) - ZP).astype(np.int8)[None] for name, t in ir.outputs}


def egress_int8(ir, tensors: Dict[str, np.ndarray]) -> np.ndarray:
    """One image's heads packed back to back in head order: the 1,209,600-byte egress for 640x640."""
    return np.concatenate([h.reshape(-1) for h in heads_int8(ir, tensors).values()])


def run_batch_egress(ir, images: np.ndarray) -> np.ndarray:
    """uint8 [B][3][H][W] -> int8 [B][egress bytes]."""
    return np.stack([egress_int8(ir, run_image(ir, im)) for im in images])


# ---------------------------------------------------------------- integer GEMM / W4A8

def srs_i8(acc, shift: int) -> np.ndarray:
    """int8 clamp of an RNE shift: the pow2 SRS epilogue in the signed domain."""
    return np.clip(rne_shift(acc, shift), -128, 127).astype(np.int8)


def exact_matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Integer a @ b as int64 through float64 BLAS: exact while every partial sum stays below 2^53
    in magnitude, which int8 operands guarantee for K < 2^38."""
    assert a.shape[-1] < (1 << 38)
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.int64)


def i8gemm_srs(a: np.ndarray, b: np.ndarray, bias: np.ndarray, shift: int) -> np.ndarray:
    """int8 A [M,K] x int8 B [N,K] (K-major) + int32 bias [N], then RNE shift and int8 clamp."""
    acc = exact_matmul(a, b.T) + bias.astype(np.int64)[None, :]
    return srs_i8(acc, shift)


def pack_int4(v: np.ndarray) -> np.ndarray:
    """Two int4 per byte along the last axis, element 2j in the LOW nibble, two's complement
    (kernels/w4a8_probe/w4a8_probe.py:197-201, tools/int4_prefill_model.py:154-179)."""
    u = (np.asarray(v).astype(np.int16) & 0xF).astype(np.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(p: np.ndarray) -> np.ndarray:
    u = np.asarray(p, dtype=np.uint8)
    lo = (u & 0xF).astype(np.int16)
    hi = (u >> 4).astype(np.int16)
    out = np.empty(u.shape[:-1] + (u.shape[-1] * 2,), dtype=np.int16)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return np.where(out >= 8, out - 16, out).astype(np.int8)


def w4a8_acc(a: np.ndarray, w_kn: np.ndarray, gpos: np.ndarray, group: int = 128) -> np.ndarray:
    """int64 accumulator sum_g (sum_{k in g} a_k w_kn) << (p_max - p_g).

    a int8 [M,K]; w_kn uint8 [K, N/2], the reference's operand (two int4 per byte along N, element
    2j in the low nibble: w4a8_probe.py:197-201, int4_prefill_model.py Int4MmulReference);
    gpos int [K/group, N] group positions, p_max their max per column. The group step is the
    engine's own (the reference kernels output the raw int32 A.B)."""
    w = unpack_int4(w_kn).astype(np.int64)                       # [K, N]
    m, k = a.shape
    pmax = gpos.max(axis=0).astype(np.int64)                      # [N]
    acc = np.zeros((m, w.shape[1]), dtype=np.int64)
    for g in range(k // group):
        part = exact_matmul(a[:, g * group:(g + 1) * group], w[g * group:(g + 1) * group])
        acc += part << (pmax - gpos[g].astype(np.int64))[None, :]
    return acc


def u8i4_i32(a_u8: np.ndarray, w_kn: np.ndarray) -> np.ndarray:
    """uint8 A [M,K] x int4 B [K,N] (packed [K, N/2], low nibble first) -> int64 [M,N], the
    reference's Int4MmulReference.execute (tools/int4_prefill_model.py:182-207) at any size."""
    return exact_matmul(np.asarray(a_u8, dtype=np.uint8).astype(np.int64), unpack_int4(w_kn).astype(np.int64))


def w4a8_srs(a, w_kn, gpos, shift: np.ndarray, group: int = 128) -> np.ndarray:
    """W4A8 output: per output column RNE shift and int8 clamp of the group-aligned accumulator."""
    acc = w4a8_acc(a, w_kn, gpos, group)
    out = np.empty(acc.shape, dtype=np.int8)
    for s in np.unique(shift):
        cols = np.nonzero(shift == s)[0]
        out[:, cols] = srs_i8(acc[:, cols], int(s))
    return out