"""CPU model of the conv/SPPF kernels' address arithmetic, for offline checks of the plan.

It walks a DevicePlan the way ``csrc/ixb_conv.cuh`` does: the same K-blocks, the same
shared-memory images of A (window / gather / stem loads) and B (the packed weights), UMMA
operands read back through the no-swizzle K-major descriptor layout
(element (r, k) at start + (r // 8) * SBO + (r % 8) * 16 + (k // 16) * LBO + k % 16), and the
same integer epilogue. It checks the host-side packing and descriptors against the oracle
without a GPU; it says nothing about the hardware beyond that layout contract.
"""
from __future__ import annotations

import numpy as np

from ignite_xdna_b200 import _lib as L
from ignite_xdna_b200.plan import DevicePlan

TILE_M = 128


def _rne(x: np.ndarray, s: int) -> np.ndarray:
    if s <= 0:
        return x << (-s)
    q = x >> s
    r = x - (q << s)
    h = 1 << (s - 1)
    return q + ((r > h) | ((r == h) & ((q & 1) == 1))).astype(np.int64)


def _operand(smem: np.ndarray, start: int, lbo: int, sbo: int, rows: int) -> np.ndarray:
    r = np.arange(rows)[:, None]
    k = np.arange(32)[None, :]
    idx = start + (r // 8) * sbo + (r % 8) * 16 + (k // 16) * lbo + (k % 16)
    return smem[idx].view(np.int8).astype(np.int64)


def _seg_params(d, s, chunk_begin):
    return dict(base=int(s.offset) + int(s.chunk_offset) * int(s.plane_stride), plane=int(s.plane_stride),
                chunk_begin=chunk_begin, chunks=(int(s.channels) + 15) // 16, H=int(s.height), W=int(s.width),
                up2=int(s.up2), P=(int(s.height) + 2) * (int(s.width) + 2))


def run_conv(arena: np.ndarray, d, batch: int, arena_bytes: int) -> None:
    info = L.conv_launch_info(d, arena_bytes, batch)
    sched = L.conv_schedule(d)
    MT = info["mt"]
    TM = 128 * MT
    mode, k, stride = d.mode, d.k, d.stride
    pad = 1 if d.s2d_in else k // 2   # the 2x2 space-to-depth taps reach one pixel back
    H, W, Ho, Wo = d.in_h, d.in_w, d.out_h, d.out_w
    n_tile = d.n_tile
    segs, chunk = [], 0
    for i in range(d.nseg):
        sp = _seg_params(d, d.seg[i], chunk)
        chunk += sp["chunks"]
        segs.append(sp)
    Wm = Wo + 1 if mode in (L.MODE_STEM, L.MODE_IM2COL) else Wo    # one spare column per output row
    if mode == L.MODE_WINDOW:
        win_origin = pad * (W + 2) + pad
        rowsA = TM + (1 if d.s2d_in else 2) * win_origin
        m_total = batch * (H + 2) * (W + 2)
    else:
        win_origin = 0
        rowsA = TM + 8 if mode in (L.MODE_STEM, L.MODE_IM2COL) else TM
        m_total = batch * Ho * Wm
    assert info["kblocks"] == len(sched) and info["rows_a"] == rowsA
    b_total = sched[-1]["b_off"] + sched[-1]["b_bytes"]
    assert (d.cout // n_tile) * b_total == d.w_bytes
    slots = max(b["nchunks"] * b["ntaps"] for b in sched)
    a_bytes = slots * rowsA * 16 + 16

    def shift_of(t):
        if mode == L.MODE_WINDOW:
            return (t // k) * (W + 2) + (t % k)
        if mode == L.MODE_STEM:
            return t & 1
        return 1 if mode == L.MODE_IM2COL and t % 3 == 2 else 0

    bias = arena[d.bias_offset:d.bias_offset + 4 * d.cout].view(np.int32).astype(np.int64)
    lut = arena[d.lut_offset:d.lut_offset + 256].view(np.int8).astype(np.int64)
    for mt in range((m_total + TM - 1) // TM):
        m0 = mt * TM
        for nt in range(d.cout // n_tile):
            acc = np.zeros((TM, n_tile), dtype=np.int64)
            for blk in sched:
                smem = np.zeros(a_bytes, dtype=np.uint8)
                # ---- A: slot s = chunk chunk0 + s // ntaps at tap tap0 + s % ntaps
                for sl in range(blk["nchunks"] * blk["ntaps"]):
                    gc = blk["chunk0"] + sl // blk["ntaps"]
                    tap = blk["tap0"] + sl % blk["ntaps"]
                    dst0 = sl * rowsA * 16
                    if mode == L.MODE_STEM:
                        # slot = image row ky (the K-block's taps 0..2), pair 0 of every M row
                        r = np.arange(rowsA)
                        m = m0 + r
                        ok = m < m_total
                        s = d.seg[0]
                        img = m // (Ho * Wm)
                        rem = m - img * Ho * Wm
                        y, x = rem // Wm, rem % Wm
                        ky = tap
                        src = s.offset + ((img * (s.height + 2) + 2 * y + ky) * (s.width + 4) + 2 * x) * 8
                        for rr in np.nonzero(ok)[0]:
                            smem[dst0 + rr * 16:dst0 + rr * 16 + 16] = arena[src[rr]:src[rr] + 16]
                        continue
                    si = [i for i, s in enumerate(segs) if s["chunk_begin"] <= gc < s["chunk_begin"] + s["chunks"]]
                    if not si:
                        continue
                    s = segs[si[-1]]
                    cbase = s["base"] + (gc - s["chunk_begin"]) * s["plane"]
                    if mode == L.MODE_WINDOW:
                        px = np.arange(rowsA)
                        m = m0 - win_origin + px
                        ok = np.ones_like(m, dtype=bool)      # one bulk copy; the plane guards are zero
                        src = cbase + m * 16
                        rows = px
                    else:
                        r = np.arange(rowsA)
                        m = m0 + r
                        ok = m < m_total
                        img = m // (Ho * Wm)
                        rem = m - img * Ho * Wm
                        y, x = rem // Wm, rem % Wm
                        if mode == L.MODE_IM2COL:
                            ky, kx = tap // 2, tap % 2           # loaded tap 2 ky + kx
                        else:
                            ky, kx = tap // k, tap % k
                        iy, ix = y * stride + ky - pad, x * stride + kx - pad
                        if s["up2"]:
                            iy, ix = iy >> 1, ix >> 1
                        src = cbase + (img * s["P"] + (iy + 1) * (s["W"] + 2) + ix + 1) * 16
                        rows = r
                    for rr, sa in zip(rows[ok], src[ok]):
                        smem[dst0 + rr * 16:dst0 + rr * 16 + 16] = arena[sa:sa + 16]
                # ---- B of this K-block, then its MMAs
                wsrc = d.w_offset + nt * b_total + blk["b_off"]
                bmem = arena[wsrc:wsrc + blk["b_bytes"]]
                for o, ((s0, _, t0), second) in enumerate(blk["ops"]):
                    a_start = s0 * rowsA + shift_of(t0)
                    lbo = (second[0] * rowsA + shift_of(second[2]) - a_start) if second is not None else 1
                    B = _operand(bmem, o * n_tile * 32, 128, 256, n_tile)
                    for blk_m in range(MT):
                        A = _operand(smem, (a_start + blk_m * 128) * 16, lbo * 16, 128, 128)
                        acc[blk_m * 128:(blk_m + 1) * 128] += A @ B.T
            # ---- epilogue
            m = m0 + np.arange(TM)
            valid = m < m_total
            if mode == L.MODE_WINDOW:
                P = (H + 2) * (W + 2)
                img = m // P
                rem = m - img * P
                yp, xp = rem // (W + 2), rem % (W + 2)
                valid &= (yp >= 1) & (yp <= H) & (xp >= 1) & (xp <= W)
                opix, oy, ox = m, yp - 1, xp - 1
            else:
                img = m // (Ho * Wm)
                rem = m - img * Ho * Wm
                oy, ox = rem // Wm, rem % Wm
                valid &= ox < Wo
                opix = img * (Ho + 2) * (Wo + 2) + (oy + 1) * (Wo + 2) + ox + 1
            co = nt * n_tile + np.arange(n_tile)
            a = acc + bias[co][None, :]
            t1 = np.clip(_rne(a, d.shift), -128, 127)
            t2 = lut[t1 + 128]
            if d.has_residual:
                r = d.residual
                rb = r.offset + r.chunk_offset * r.plane_stride
                ra = rb + (co[None, :] // 16) * r.plane_stride + opix[:, None] * 16 + (co[None, :] % 16)
                rv = arena[np.where(valid[:, None], ra, 0)].view(np.int8).astype(np.int64)
                t2 = np.clip(_rne((t2 << d.res_lsh_main) + (rv << d.res_lsh_res), d.res_shift), -128, 127)
            out = t2.astype(np.int8).view(np.uint8)
            for rr in np.nonzero(valid)[0]:
                if not d.out_nchw:
                    ob = d.out.offset + d.out.chunk_offset * d.out.plane_stride
                    for j in range(n_tile // 16):
                        if d.out2_kind == L.OUT2_S2D_ONLY:
                            break
                        a0 = ob + (nt * n_tile // 16 + j) * d.out.plane_stride + opix[rr] * 16
                        arena[a0:a0 + 16] = out[rr, 16 * j:16 * j + 16]
                    if d.out2_kind in (L.OUT2_S2D, L.OUT2_S2D_ONLY):  # the space-to-depth view
                        u = d.out2
                        ph = (oy[rr] % 2) * 2 + ox[rr] % 2
                        pix = img[rr] * (u.height + 2) * (u.width + 2) + (oy[rr] // 2 + 1) * (u.width + 2) + ox[rr] // 2 + 1
                        for j in range(n_tile // 16):
                            a0 = u.offset + (ph * (d.cout // 16) + nt * n_tile // 16 + j) * u.plane_stride + pix * 16
                            arena[a0:a0 + 16] = out[rr, 16 * j:16 * j + 16]
                    if d.out2_kind == L.OUT2_UP2:  # the 2x2-replicated copy at twice the resolution
                        u = d.out2
                        W2, P2 = u.width + 2, (u.height + 2) * (u.width + 2)
                        for j in range(n_tile // 16):
                            base = u.offset + (nt * n_tile // 16 + j) * u.plane_stride
                            for dy in (0, 1):
                                for dx in (0, 1):
                                    a0 = base + (img[rr] * P2 + (2 * oy[rr] + 1 + dy) * W2 + 2 * ox[rr] + 1 + dx) * 16
                                    arena[a0:a0 + 16] = out[rr, 16 * j:16 * j + 16]
                else:
                    plane = Ho * Wo
                    e = d.egress_offset + img[rr] * d.egress_image_bytes + oy[rr] * Wo + ox[rr]
                    keep = co < (d.egress_channels or d.cout)
                    arena[e + co[keep] * plane] = out[rr][keep]


def run_pool(arena: np.ndarray, pd, batch: int) -> None:
    s = pd.inp
    H, W, C = s.height, s.width, s.channels
    P = (H + 2) * (W + 2)
    for c in range(C // 16):
        for b in range(batch):
            base = s.offset + (s.chunk_offset + c) * s.plane_stride + b * P * 16
            v = arena[base:base + P * 16].view(np.int8).reshape(H + 2, W + 2, 16)
            cur = v[1:-1, 1:-1].astype(np.int64)
            for kk in range(3):
                p = np.full((H + 4, W + 4, 16), -128, dtype=np.int64)
                p[2:-2, 2:-2] = cur
                nxt = np.full((H, W, 16), -128, dtype=np.int64)
                for dy in range(5):
                    for dx in range(5):
                        nxt = np.maximum(nxt, p[dy:dy + H, dx:dx + W])
                o = pd.out[kk]
                ob = o.offset + (o.chunk_offset + c) * o.plane_stride + b * P * 16
                ov = arena[ob:ob + P * 16].view(np.int8).reshape(H + 2, W + 2, 16)
                ov[1:-1, 1:-1] = nxt.astype(np.int8)
                cur = nxt


def run_network(dp: DevicePlan, images: np.ndarray) -> np.ndarray:
    """uint8 images [B,3,H,W] -> int8 egress [B, bytes], through the modelled kernels."""
    batch = images.shape[0]
    arena = np.zeros(dp.arena_bytes, dtype=np.uint8)
    arena[dp.const_offset:dp.const_offset + dp.const_blob.size] = dp.const_blob
    lut = arena[dp.input_lut_offset:dp.input_lut_offset + 256].view(np.int8)
    s = dp.input_store
    for b in range(batch):
        n = (s.height + 2) * (s.width + 4) * 8
        base = s.offset + b * n
        v = arena[base:base + n].view(np.int8).reshape(s.height + 2, s.width + 4, 8)
        v[1:-1, 1:s.width + 1, :3] = lut[images[b].transpose(1, 2, 0)]
    if dp.input_s2d_store is not None:   # the image's space-to-depth view: byte ph * 3 + c
        v2 = dp.input_s2d_store
        P2 = (v2.height + 2) * (v2.width + 2)
        for b in range(batch):
            q = lut[images[b]]                                   # [3, H, W]
            view = arena[v2.offset + b * P2 * 16:v2.offset + (b + 1) * P2 * 16].view(np.int8)
            view = view.reshape(v2.height + 2, v2.width + 2, 16)
            for ph in range(4):
                ry, rx = divmod(ph, 2)
                view[1:-1, 1:-1, 3 * ph:3 * ph + 3] = q[:, ry::2, rx::2].transpose(1, 2, 0)
    convs = [c.desc for c in dp.convs]
    for kind, idx in dp.ops:
        if (kind & 0xFF) == L.OP_CONV:
            run_conv(arena, convs[idx], batch, dp.arena_bytes)
        else:
            run_pool(arena, dp.pools[idx][1], batch)
    e = arena[dp.egress_offset:dp.egress_offset + batch * dp.egress_image_bytes]
    return e.view(np.int8).reshape(batch, dp.egress_image_bytes).copy()
