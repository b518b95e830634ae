"""Host-side plan: packed weights, descriptors and storage, checked through the CPU kernel model."""
import numpy as np
import pytest

import ixb_oracle as O
import kernel_model as KM
from ignite_xdna_b200 import _lib as L
from ignite_xdna_b200 import build_yolov8, random_images
from ignite_xdna_b200.plan import build_plan, input_lut_t


@pytest.mark.parametrize("imgsz,batch,sms", [(64, 2, None), (96, 1, None), (64, 2, "1"), (96, 1, "2")])
def test_kernel_model_matches_oracle(imgsz, batch, sms, monkeypatch):
    """sms forces the launch planner's SM count, so small inputs take the 256/512-row tiles."""
    if sms:
        monkeypatch.setenv("IXB_SM_COUNT", sms)
    ir = build_yolov8("n", imgsz=imgsz)
    dp = build_plan(ir, batch)
    imgs = random_images(batch, imgsz, seed=11)
    assert np.array_equal(KM.run_network(dp, imgs), O.run_batch_egress(ir, imgs))


def test_kernel_model_with_im2col_stride2_matches_oracle(monkeypatch):
    """IXB_S2D=0: the stride-2 3x3 convs load their A operand with TMA im2col (IM2COL mode)."""
    monkeypatch.setenv("IXB_S2D", "0")
    ir = build_yolov8("n", imgsz=64)
    dp = build_plan(ir, 2)
    assert sum(c.mode == L.MODE_IM2COL for c in dp.convs) == 6 and not dp.s2d_stores
    imgs = random_images(2, 64, seed=13)
    assert np.array_equal(KM.run_network(dp, imgs), O.run_batch_egress(ir, imgs))


def test_kernel_model_with_gathered_upsample_matches_oracle(monkeypatch):
    """IXB_UP2=0: the concat convs gather the upsampled tensors (GATHER mode)."""
    monkeypatch.setenv("IXB_UP2", "0")
    ir = build_yolov8("n", imgsz=64)
    dp = build_plan(ir, 2)
    assert sum(c.mode == L.MODE_GATHER for c in dp.convs) == 2 and not dp.upsampled_stores
    imgs = random_images(2, 64, seed=12)
    assert np.array_equal(KM.run_network(dp, imgs), O.run_batch_egress(ir, imgs))


def test_pose_plan_pads_ragged_channels_and_matches_oracle():
    """One-class heads and 51-channel keypoint branches: storage and output channels round up to
    whole 16-channel chunks (zero weights and bias), the heads write only their real channels."""
    ir = build_yolov8("n", imgsz=64, task="pose")
    dp = build_plan(ir, 2)
    by_out = {c.layer.output: c.desc for c in dp.convs}
    kpt = ir.tensors[dict(ir.outputs)["p3_kpt"]]
    assert kpt.channels == 51 and by_out[kpt.name].cout == 64 and by_out[kpt.name].egress_channels == 51
    cls = dict(ir.outputs)["p4_cls"]
    assert by_out[cls].cout == 16 and by_out[cls].egress_channels == 1
    mid = [c for c in dp.convs if c.layer.cout == 51 and c.layer.output not in dict(ir.outputs).values()]
    assert mid and all(dp.stores[c.layer.output].channels == 64 for c in mid)
    assert dp.egress_image_bytes == sum(ir.tensors[t].channels * ir.tensors[t].height * ir.tensors[t].width
                                        for _, t in ir.outputs)
    imgs = random_images(2, 64, seed=11)
    assert np.array_equal(KM.run_network(dp, imgs), O.run_batch_egress(ir, imgs))


@pytest.mark.parametrize("task", ["detect", "pose"])
def test_branch_schedule_is_a_valid_order(task):
    """Every op once; each op after all producers of what it reads; the members of a branch group
    neither read nor write each other's outputs; without branches the order is the graph's."""
    ir = build_yolov8("n", imgsz=64, task=task)
    dp = build_plan(ir, 2, branches=True)
    plain = build_plan(ir, 2, branches=False)
    assert sorted((k & 0xFF, i) for k, i in dp.ops) == sorted(plain.ops)
    assert not any(k & L.OP_WITH_PREV for k, _ in plain.ops)

    def rw(k, i):
        if (k & 0xFF) == L.OP_CONV:
            layer = dp.convs[i].layer
            r = {s.tensor for s in layer.inputs} | ({layer.residual.tensor} if layer.residual else set())
            return r, {layer.output}
        chain = dp.pools[i][0]
        return {chain[0].input.tensor}, {p.output for p in chain}
    groups = []
    for k, i in dp.ops:
        if k & L.OP_WITH_PREV:
            groups[-1].append((k, i))
        else:
            groups.append([(k, i)])
    written = {ir.input}
    for g in groups:
        # every member reads only what earlier groups wrote (so nothing of its own group)
        for k, i in g:
            assert rw(k, i)[0] <= written
        written |= set().union(*[rw(k, i)[1] for k, i in g])
    sizes, run = [], 0
    for k, _ in dp.ops:
        run = run + 1 if k & L.OP_WITH_PREV else 1
        sizes.append(run)
    assert max(sizes) >= 2 and max(sizes) <= L.MAX_BRANCHES


def test_input_table_is_reference_lut():
    lut = input_lut_t(2.0 ** -7)
    ref = O.input_lut(2.0 ** -7).astype(np.int16) - 128
    assert np.array_equal(lut.astype(np.int16), ref)
    assert lut.min() == 0 and lut.max() == 127


@pytest.mark.parametrize("variant", ["n", "s", "m"])
def test_plan_storage_is_disjoint_and_aligned(variant):
    ir = build_yolov8(variant)
    dp = build_plan(ir, 64)
    spans = {}
    for name, st in dp.stores.items():
        nch = sum(t.channels for n2, t in ir.tensors.items() if n2 in dp.stores and dp.stores[n2].offset == st.offset) // 16
        start = st.offset - st.guard * 16
        spans[start] = nch * st.plane_stride
        assert st.offset % 16 == 0 and st.plane_stride % ((st.height + 2) * (st.width + 2) * 16) == 0
        assert st.plane_stride >= (64 * (st.height + 2) * (st.width + 2) + 2 * st.guard) * 16
    spans[dp.images_offset] = 64 * 3 * dp.img_h * dp.img_w
    spans[dp.input_store.offset] = 64 * (dp.img_h + 2) * (dp.img_w + 4) * 8
    spans[dp.egress_offset] = 64 * dp.egress_image_bytes
    assert len(dp.extra_images_offsets) == len(dp.extra_egress_offsets) == 2
    for a, e in zip(dp.extra_images_offsets, dp.extra_egress_offsets):
        spans[a] = 64 * 3 * dp.img_h * dp.img_w
        spans[e] = 64 * dp.egress_image_bytes
    spans[dp.const_offset] = dp.const_blob.size
    assert len(dp.upsampled_stores) == 2  # the top-down path's two upsampled tensors
    for name, st in dp.upsampled_stores.items():
        t = ir.tensors[name]
        assert (st.height, st.width) == (2 * t.height, 2 * t.width)
        spans[st.offset - st.guard * 16] = st.channels // 16 * st.plane_stride
    assert not any(c.mode in (L.MODE_GATHER, L.MODE_IM2COL) for c in dp.convs)
    assert sum(c.desc.out2_kind == L.OUT2_UP2 for c in dp.convs) == 2
    assert sum(c.s2d for c in dp.convs) == 6 and len(dp.s2d_stores) == 6
    for name, st in dp.s2d_stores.items():
        t = ir.tensors[name]
        assert (st.height, st.width, st.channels) == (t.height // 2, t.width // 2, 4 * t.channels)
        spans[st.offset - st.guard * 16] = st.channels // 16 * st.plane_stride
    iv = sorted(spans.items())
    for (a, n), (b, _) in zip(iv, iv[1:]):
        assert a + n <= b
    assert iv[-1][0] + iv[-1][1] <= dp.arena_bytes
    assert dp.egress_image_bytes == 1_209_600


def _sched(mode, k, cin, cp, n_tile=32):
    d = L.ConvDesc()
    d.mode, d.k, d.stride, d.n_tile, d.cp, d.cin, d.cout, d.nseg = mode, k, 1, n_tile, cp, cin, n_tile, 1
    d.seg[0].channels = cin
    return L.conv_schedule(d)


@pytest.mark.parametrize("mode", [L.MODE_WINDOW, L.MODE_GATHER, L.MODE_IM2COL])
@pytest.mark.parametrize("k,cin,cp", [(3, 80, 1), (1, 384, 4), (3, 576, 2), (1, 48, 2), (3, 16, 1), (1, 16, 1),
                                      (3, 48, 1), (1, 80, 4)])
def test_schedule_covers_every_tap_and_chunk_once(mode, k, cin, cp):
    if mode == L.MODE_IM2COL and k != 3:
        pytest.skip("IM2COL is the 3x3 stride-2 conv")
    if mode == L.MODE_GATHER and k != 1:
        pytest.skip("GATHER is the 1x1 conv over an upsampled concat")
    nchunks = (cin + 15) // 16
    seen = []
    for blk in _sched(mode, k, cin, cp):
        nslots = blk["nchunks"] * blk["ntaps"]
        for first, second in blk["ops"]:
            for half in (first, second):
                if half is None:
                    continue
                slot, chunk, tap = half
                assert slot < nslots
                if mode == L.MODE_IM2COL:     # the slot's loaded tap 2 ky + kx; kx = 2 reads kx = 0
                    assert chunk == blk["chunk0"] + slot // blk["ntaps"]
                    lt = blk["tap0"] + slot % blk["ntaps"]
                    assert tap // 3 == lt // 2 and (tap % 3 == lt % 2 or (tap % 3 == 2 and lt % 2 == 0))
                elif mode != L.MODE_WINDOW:   # the slot's loaded (chunk, tap) is the half's
                    assert chunk == blk["chunk0"] + slot // blk["ntaps"]
                    assert tap == blk["tap0"] + slot % blk["ntaps"]
                else:
                    assert chunk == blk["chunk0"] + slot
                seen.append((tap, chunk))
    assert sorted(seen) == sorted((t, c) for t in range(k * k) for c in range(nchunks))


def test_odd_chunk_taps_are_paired():
    """A 16-channel 3x3 conv needs 5 MMAs per 128 pixels, not 9, window or im2col."""
    blocks = _sched(L.MODE_WINDOW, 3, 16, 1)
    assert len(blocks) == 1 and len(blocks[0]["ops"]) == 5
    blocks = _sched(L.MODE_WINDOW, 3, 80, 1)
    assert sum(len(b["ops"]) for b in blocks) == 2 * 9 + 5
    blocks = _sched(L.MODE_IM2COL, 3, 16, 1)
    assert sum(len(b["ops"]) for b in blocks) == 5


def test_fast_division_formula_is_exact():
    """The kernels divide pixel indices (< 2^31) by invariant divisors with
    q = (umulhi(n, m) + n) >> s, m = floor(2^32 (2^s - d) / d) + 1, s = ceil(log2 d)."""
    rng = np.random.default_rng(0)
    divisors = list(range(1, 2000)) + [162 * 162, 322 * 322, 642 * 642, 6400, 25600, 102400, 1 << 20, 12345679]
    for d in divisors:
        s = int(np.ceil(np.log2(d))) if d > 1 else 0
        while (1 << s) < d:
            s += 1
        m = ((1 << 32) * ((1 << s) - d)) // d + 1
        n = np.concatenate([rng.integers(0, 2 ** 31, 4000, dtype=np.int64), np.arange(0, 3 * d + 5),
                            np.array([2 ** 31 - 1, 2 ** 31 - 2, d * (2 ** 31 // d) - 1])]).astype(np.uint64)
        q = (((n * np.uint64(m)) >> np.uint64(32)) + n) >> np.uint64(s)
        assert np.array_equal(q, n // np.uint64(d)), d
