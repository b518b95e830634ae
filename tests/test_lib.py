"""The C ABI library: it loads, exports every declared entry point, and its host-side checks
refuse descriptors that would reach outside the arena (no GPU needed: validation runs first)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from ignite_xdna_b200 import _lib as L
from ignite_xdna_b200 import build_yolov8
from ignite_xdna_b200.plan import build_plan

HEADER = Path(__file__).resolve().parent.parent / "include" / "ixb200.h"


def declared():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(ixb_\w+)\(", txt, re.M)))


def test_header_declares_what_binding_binds():
    assert declared() == L.exported_symbols()


def test_library_loads_and_exports_every_symbol():
    lib = L.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.ixb_version() == L.API_VERSION


def _desc():
    ir = build_yolov8("n", imgsz=64)
    dp = build_plan(ir, 2)
    return dp, [c.desc for c in dp.convs]


def test_valid_descriptor_passes_checks_until_launch():
    dp, descs = _desc()
    lib = L.load()
    # arena pointer is a dummy: validation runs on the host before any CUDA call
    rc = lib.ixb_conv_layer(C.byref(descs[3]), C.c_void_p(0x10000), dp.arena_bytes, 2, None)
    # either launched (GPU present) or failed in CUDA, never rejected as invalid
    assert rc != -1 or "arena" not in lib.ixb_last_error().decode()


@pytest.mark.parametrize("mutate,needle", [
    (lambda d, n: setattr(d.out, "offset", n), "arena"),
    (lambda d, n: setattr(d.seg[0], "offset", n - 64), "arena"),
    (lambda d, n: setattr(d, "w_offset", n), "weights"),
    (lambda d, n: setattr(d, "shift", 48), "shift"),
    (lambda d, n: setattr(d, "shift", -32), "shift"),
    (lambda d, n: setattr(d.seg[0], "plane_stride", d.seg[0].plane_stride + 8), "misaligned"),
    (lambda d, n: setattr(d.seg[0], "guard", 0), "guard"),
    (lambda d, n: setattr(d.out, "chunk_offset", 10 ** 6), "arena"),
    (lambda d, n: setattr(d, "n_tile", 24), "n_tile"),
    (lambda d, n: setattr(d, "cin", d.cin + 16), "cin"),
])
def test_host_checks_refuse_out_of_bounds_descriptors(mutate, needle):
    dp, descs = _desc()
    lib = L.load()
    # a WINDOW 1x1 (the first conv past the stem block) with a plain output view
    d = L.ConvDesc.from_buffer_copy(next(x for x in descs[5:] if x.mode == L.MODE_WINDOW and x.k == 1
                                         and x.out2_kind == L.OUT2_NONE and not x.out_nchw))
    mutate(d, dp.arena_bytes)
    rc = lib.ixb_conv_layer(C.byref(d), C.c_void_p(0x10000), dp.arena_bytes, 2, None)
    assert rc == -1
    assert needle in lib.ixb_last_error().decode()


def test_batch_beyond_plan_is_refused():
    dp, descs = _desc()
    lib = L.load()
    rc = lib.ixb_conv_layer(C.byref(descs[5]), C.c_void_p(0x10000), dp.arena_bytes, 100000, None)
    assert rc == -1 and any(w in lib.ixb_last_error().decode() for w in ("arena", "overlap", "pixel"))


def _create(dp, ops):
    """ixb_session_create on the plan with ``ops`` as its op list (no arena: validation only)."""
    from ignite_xdna_b200.plan import c_plan
    p = c_plan(dp)
    arr = (L.Op * len(ops))(*[L.Op(k, i) for k, i in ops])
    p.ops, p.n_ops = arr, len(ops)
    lib = L.load()
    h = C.c_void_p()
    rc = lib.ixb_session_create(C.byref(p), 0, None, 0, C.byref(h))
    if rc == 0:
        lib.ixb_session_destroy(h)
    return rc, lib.ixb_last_error().decode()


def test_branch_groups_pass_the_hazard_check():
    """The planner's branch groups are accepted: session creation gets past the op checks (to the
    first CUDA call, on a machine without a GPU)."""
    dp = build_plan(build_yolov8("n", imgsz=64), 2, branches=True)
    assert any(k & L.OP_WITH_PREV for k, _ in dp.ops)
    rc, msg = _create(dp, dp.ops)
    assert rc == 0 or "branch group" not in msg and "op list" not in msg


def test_branch_group_with_a_dependency_is_refused():
    dp, _ = _desc()
    ops = [(k & 0xFF, i) for k, i in dp.ops]
    # a conv joined to its own producer: reads what the other member writes
    j = next(n for n in range(1, len(ops)) if ops[n][0] == L.OP_CONV and ops[n - 1][0] == L.OP_CONV)
    ops[j] = (ops[j][0] | L.OP_WITH_PREV, ops[j][1])
    rc, msg = _create(dp, ops)
    assert rc == L.IXB_ERR_INVALID and "branch group" in msg
    ops = [(k & 0xFF, i) for k, i in dp.ops]
    ops[0] = (ops[0][0] | L.OP_WITH_PREV, ops[0][1])
    assert _create(dp, ops)[0] == L.IXB_ERR_INVALID


def test_gemm_plan_fits_the_hardware():
    import ctypes as C
    lib = L.load()
    for M, N, K in [(256, 256, 256), (8192, 8192, 8192), (1000, 48, 144), (2 * 160 * 160 * 64, 32, 288),
                    (512, 11008, 4096), (129, 16, 16), (128, 512, 65536)]:
        info = (C.c_int32 * 10)()
        assert lib.ixb_gemm_plan_info(M, N, K, 0, info, 10) == 0, (M, N, K)
        bn, mt, mtiles, ntiles, kblocks, stages, grid, smem, tcols, stage_bytes = list(info)
        assert bn % 16 == 0 and 16 <= bn <= 256 and N % 16 == 0
        assert mt * 128 * mtiles >= M and bn * ntiles >= N and kblocks * 128 >= K
        # two accumulators of MT x BN columns, or one 256 x 256 tile filling TMEM
        assert (2 * mt * bn <= tcols or (mt, bn) == (2, 256) and tcols == 512) and tcols <= 512
        assert tcols & (tcols - 1) == 0
        assert stages >= 2 and smem <= 227 * 1024 and stage_bytes * stages + 1024 + 256 <= smem
        assert 1 <= grid <= 148


def test_gemm_refuses_bad_shapes_without_touching_the_gpu():
    import ctypes as C
    lib = L.load()
    info = (C.c_int32 * 10)()
    for M, N, K in [(0, 16, 16), (16, 24, 16), (16, 16, 8), (16, 16, 65552)]:
        assert lib.ixb_gemm_plan_info(M, N, K, 0, info, 10) == L.IXB_ERR_INVALID
    x = C.c_void_p(16)
    assert lib.ixb_i8gemm_srs(x, x, x, x, 16, 16, 16, 24, None) == L.IXB_ERR_INVALID
    assert lib.ixb_i8gemm_srs(None, x, x, x, 16, 16, 16, 3, None) == L.IXB_ERR_INVALID
    assert lib.ixb_i8gemm_i32(C.c_void_p(17), x, x, 16, 16, 16, None) == L.IXB_ERR_INVALID


def test_w4a8_plan_and_refusals():
    import ctypes as C
    lib = L.load()
    info = (C.c_int32 * 10)()
    for M, N, K in [(512, 11008, 4096), (512, 4096, 11008), (1, 4096, 128), (200, 64, 256)]:
        assert lib.ixb_gemm_plan_info(M, N, K, 1, info, 10) == 0
        bn, mt, mtiles, ntiles, kblocks, stages, grid, smem, tcols, stage_bytes = list(info)
        # two accumulators of MT x BN columns, or one of up to 512 when every CTA has one tile
        one_wave = mtiles * ntiles <= grid
        assert (mt * bn <= 256 or (one_wave and mt * bn <= 512)) and bn % 16 == 0 and bn <= 256
        assert kblocks * 128 == K and mt * 128 * mtiles >= M
        nacc = 2 if 2 * mt * bn <= 512 else 1
        assert stages >= 2 and smem <= 227 * 1024 and nacc * mt * bn <= tcols <= 512
    assert lib.ixb_gemm_plan_info(512, 64, 200, 1, info, 10) == L.IXB_ERR_INVALID   # K not a whole group
    nbytes = C.c_uint64()
    assert lib.ixb_w4a8_image_bytes(4096, 11008, C.byref(nbytes)) == 0
    assert nbytes.value == 11008 * 2048 + 11008 * 32
    assert lib.ixb_w4a8_image_bytes(100, 16, C.byref(nbytes)) == L.IXB_ERR_INVALID
    x = C.c_void_p(16)
    assert lib.ixb_w4a8_gemv(x, x, x, x, 24, 128, None) == L.IXB_ERR_INVALID
    assert lib.ixb_w4a8_gemm(x, x, None, x, 16, 16, 128, None) == L.IXB_ERR_INVALID


def test_window_tiles_shrink_to_fit_smaller_guards():
    """A WINDOW view planned with smaller plane guards (the earlier rule, 1024 + 2 (W + 3) + 64)
    still builds: the launch planner skips tile sizes whose window copies would pass the guard."""
    ir = build_yolov8("n", imgsz=640)
    dp = build_plan(ir, 64)
    stem = L.ConvDesc.from_buffer_copy(dp.convs[0].desc)      # 16 channels: takes 2048-row tiles
    full = L.conv_launch_info(stem, dp.arena_bytes, 64)
    assert full["tile_rows"] == 2048
    small = L.ConvDesc.from_buffer_copy(stem)
    for i in range(small.nseg):
        small.seg[i].guard = 1024 + 2 * (small.in_w + 3) + 64
    info = L.conv_launch_info(small, dp.arena_bytes, 64)
    assert info["tile_rows"] < 2048
    end = info["m_tiles"] * info["tile_rows"] + (small.in_w + 2) + 1
    assert end <= 64 * (small.in_h + 2) * (small.in_w + 2) + small.seg[0].guard
