"""SiLU as a 256-entry int8 table: the four-line piecewise-linear sigmoid epilogue.

This is the model-build step that turns a SiLU site with linear-output scale s1 and
activation scale s2 into the table the conv epilogue indexes. It restates, in this
package's own code, the fitting procedure of the reference's
``src/ignite_xdna/compiler/silu_sigmoid.py``:

* the integer epilogue (``engine_emulator.sigmoid_epilogue``, engine_emulator.py:179-192):
  ``u = |t|; g = clip(min_i sat16(rne((u*A_i + B_i) >> S)), 0, 64);
  y = sat16(rne(((t << 6) + u*g) >> YSH))`` with ``YSH = 7 - log2 s1 + log2 s2``;
* a float minimax chord fit of ``sigmoid(u) - 0.5`` on ``[0, 128*s1]`` by breakpoint
  search (silu_sigmoid.py:67-104), converted to integers at the largest shift S in
  [6, 14] whose slopes fit int16 (silu_sigmoid.py:107-111);
* a coordinate descent over the integer constants minimising (max, mean) output-LSB
  error against ``clip(round(silu(t*s1)/s2))`` (silu_sigmoid.py:112-128).

The float search must take the same steps in the same order as the reference for the
tables to come out byte-identical; the golden fixtures under ``tests/golden`` pin them.
"""
from __future__ import annotations

import math
from typing import Dict, List, Sequence, Tuple

import numpy as np

from .graph import SigmoidFit

N_LINES = 4
_T = np.arange(-128, 128, dtype=np.int64)
_CACHE: Dict[Tuple[float, float], SigmoidFit] = {}


def rne_shift(x, s: int) -> np.ndarray:
    """Arithmetic shift right by s with round-half-to-even; s <= 0 shifts left."""
    x = np.asarray(x, dtype=np.int64)
    if s <= 0:
        return x << (-s)
    q = x >> s
    r = x - (q << s)
    h = np.int64(1) << (s - 1)
    return q + ((r > h) | ((r == h) & ((q & 1) == 1))).astype(np.int64)


def sat16(x) -> np.ndarray:
    return np.clip(np.asarray(x, dtype=np.int64), -32768, 32767)


def _exp2_exact(scale: float) -> int:
    e = math.log2(scale)
    if abs(e - round(e)) > 1e-9:
        raise ValueError(f"scale {scale} is not a power of two")
    return int(round(e))


def output_shift(s1: float, s2: float) -> int:
    return 7 - _exp2_exact(s1) + _exp2_exact(s2)


def exact_silu_t(s1: float, s2: float) -> np.ndarray:
    """The exactly quantized SiLU over t = -128..127."""
    x = _T * s1
    return np.clip(np.round(x / (1 + np.exp(-x)) / s2), -128, 127).astype(np.int64)


def _gate(lines: Sequence[Sequence[int]], s: int) -> np.ndarray:
    u = np.abs(_T)
    g = np.minimum.reduce([sat16(rne_shift(u * a + b, s)) for a, b in lines])
    return np.clip(g, 0, 64)


def epilogue_t(lines: Sequence[Sequence[int]], s: int, ysh: int) -> np.ndarray:
    """The integer epilogue over t = -128..127, clamped to int8."""
    y = sat16(rne_shift((_T << 6) + np.abs(_T) * _gate(lines, s), ysh))
    return np.clip(y, -128, 127)


def _err(y: np.ndarray, ref: np.ndarray) -> Tuple[int, float]:
    d = np.abs(y - ref)
    return int(d.max()), float(d.mean())


def _chords(bp: Sequence[float], grid: np.ndarray, target: np.ndarray, k: int):
    """Chord lines through consecutive breakpoints, centred on their error band."""
    lines = []
    for i in range(k):
        u0, u1 = bp[i], bp[i + 1]
        g0 = 1 / (1 + np.exp(-u0)) - 0.5
        g1 = 1 / (1 + np.exp(-u1)) - 0.5
        a = (g1 - g0) / (u1 - u0)
        lines.append((a, g0 - a * u0))
    approx = np.minimum.reduce([a * grid + b for a, b in lines] + [np.full_like(grid, 0.5)])
    e = target - approx
    mid = (e.max() + e.min()) / 2
    lines = [(a, b + mid) for a, b in lines]
    approx = np.minimum.reduce([a * grid + b for a, b in lines] + [np.full_like(grid, 0.5)])
    return lines, float(np.abs(target - approx).max())


def _float_fit(k: int, r: float):
    grid = np.linspace(0, r, 4001)
    target = 1 / (1 + np.exp(-grid)) - 0.5
    bp = list(np.linspace(0, min(r, 8.0), k + 1))
    best_lines, best = _chords(bp, grid, target, k)
    for _ in range(60):
        moved = False
        for i in range(1, k + 1):
            for step in (0.2, 0.05, 0.01):
                for d in (-step, step):
                    cand = list(bp)
                    cand[i] += d
                    if not all(cand[j] < cand[j + 1] for j in range(k)) or cand[-1] > r:
                        continue
                    lines, e = _chords(cand, grid, target, k)
                    if e < best - 1e-9:
                        bp, best, best_lines, moved = cand, e, lines, True
        if not moved:
            break
    return best_lines


def _integer_fit(s1: float, s2: float, k: int):
    ref = exact_silu_t(s1, s2)
    ysh = output_shift(s1, s2)
    fl = _float_fit(k, 128 * s1)
    s = max(v for v in range(6, 15) if all(abs(round(128 * a * s1 * (1 << v))) < 1 << 15 for a, _ in fl))
    lines: List[List[int]] = [[int(round(128 * a * s1 * (1 << s))), int(round(128 * b * (1 << s)))] for a, b in fl]
    best = _err(epilogue_t(lines, s, ysh), ref)
    steps = [1 << e for e in range(s, -1, -1)]
    moved = True
    while moved:
        moved = False
        for i in range(k):
            for j in range(2):
                for st in steps:
                    for sgn in (-1, 1):
                        cand = [list(l) for l in lines]
                        cand[i][j] += sgn * st
                        if j == 0 and not 0 < cand[i][j] < 1 << 15:
                            continue
                        sc = _err(epilogue_t(cand, s, ysh), ref)
                        if sc < best:
                            lines, best, moved = cand, sc, True
    return lines, s, best


def table_u8(lines: Sequence[Sequence[int]], s: int, ysh: int) -> np.ndarray:
    """The epilogue as a uint8 table indexed by the uint8 linear output q1 (zero point 128)."""
    return (epilogue_t(lines, s, ysh) + 128).astype(np.uint8)


def fit_sigmoid(s1: float, s2: float) -> SigmoidFit:
    """Sigmoid-epilogue constants and table for a SiLU with scales (s1, s2); cached per pair."""
    key = (float(s1), float(s2))
    fit = _CACHE.get(key)
    if fit is None:
        ysh = output_shift(s1, s2)
        if ysh < 0:
            raise ValueError(f"SiLU output scale {s2} is finer than the epilogue supports for input scale {s1}")
        lines, s, (mx, mean) = _integer_fit(s1, s2, N_LINES)
        for a, b in lines:
            if not (0 <= a < 1 << 15 and -(1 << 31) <= b < 1 << 31):
                raise ValueError(f"sigmoid line ({a}, {b}) does not fit an int16 slope and an int32 intercept")
        fit = SigmoidFit(tuple((int(a), int(b)) for a, b in lines), int(s), int(ysh),
                         table_u8(lines, s, ysh), mx, mean)
        _CACHE[key] = fit
    return fit
