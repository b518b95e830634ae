"""W4A8 on a B200 through the C ABI against the oracle (numpy int64), bit-exact: the weight image
from the reference's packed operand, the tcgen05 prefill GEMM and the split-K GEMV, at the MLP
projection shapes and at small and ragged ones; a group spread above 4 is refused."""
import ctypes as C

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make_case(M, N, K, seed, spread=3):
    rng = np.random.default_rng(seed)
    a = np.clip(np.rint(rng.normal(0, 24, size=(M, K))), -127, 127).astype(np.int8)
    w = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    gpos = (5 + rng.integers(0, spread + 1, size=(K // 128, N))).astype(np.int8)
    shift = rng.integers(6, 14, size=N).astype(np.int32)
    return a, O.pack_int4(w), gpos, shift


def prepare(w_kn, gpos, K, N):
    import torch
    lib = L.load()
    nbytes = C.c_uint64()
    L.check(lib.ixb_w4a8_image_bytes(K, N, C.byref(nbytes)))
    img = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    dw, dg = _dev(w_kn), _dev(gpos)
    rc = lib.ixb_w4a8_prepare(C.c_void_p(dw.data_ptr()), C.c_void_p(dg.data_ptr()), K, N, C.c_void_p(img.data_ptr()),
                              None)
    return rc, img


def run(a, w_kn, gpos, shift, gemv=False):
    import torch
    lib = L.load()
    M, K = a.shape
    N = shift.size
    rc, img = prepare(w_kn, gpos, K, N)
    L.check(rc)
    da, ds = _dev(a), _dev(shift)
    out = torch.empty((M, N), dtype=torch.int8, device="cuda")
    if gemv:
        L.check(lib.ixb_w4a8_gemv(C.c_void_p(da.data_ptr()), C.c_void_p(img.data_ptr()), C.c_void_p(ds.data_ptr()),
                                  C.c_void_p(out.data_ptr()), N, K, None))
    else:
        L.check(lib.ixb_w4a8_gemm(C.c_void_p(da.data_ptr()), C.c_void_p(img.data_ptr()), C.c_void_p(ds.data_ptr()),
                                  C.c_void_p(out.data_ptr()), M, N, K, None))
    torch.cuda.synchronize()
    L.check(lib.ixb_device_error(C.byref(C.c_int())))
    return out.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(512, 11008, 4096), (512, 4096, 11008), (128, 256, 512), (200, 48, 384),
                                   (37, 4096, 1024), (640, 64, 128)])
def test_w4a8_gemm_matches_oracle(M, N, K):
    a, w, gpos, shift = make_case(M, N, K, seed=M + N + K)
    assert np.array_equal(run(a, w, gpos, shift), O.w4a8_srs(a, w, gpos, shift))


@pytest.mark.parametrize("N,K", [(4096, 11008), (11008, 4096), (16, 128), (48, 1152), (272, 640), (160, 256),
                                 (400, 16384), (32, 65536)])
def test_w4a8_gemv_matches_oracle(N, K):
    a, w, gpos, shift = make_case(1, N, K, seed=N + K)
    assert np.array_equal(run(a, w, gpos, shift, gemv=True), O.w4a8_srs(a, w, gpos, shift))


def test_w4a8_extremes():
    """-128 / -8 operands at the largest group shifts: the int32 accumulator's worst case."""
    M, N, K = 256, 64, 4096
    a = np.full((M, K), -128, dtype=np.int8)
    a[1::2] = 127
    w = np.full((K, N), -8, dtype=np.int8)
    w[:, 1::2] = 7
    gpos = np.full((K // 128, N), 3, dtype=np.int8)
    gpos[0] = 7                       # every other group shifted by the maximum 4
    shift = np.full(N, 23, dtype=np.int32)
    wk = O.pack_int4(w)
    ref = O.w4a8_srs(a, wk, gpos, shift)
    assert np.array_equal(run(a, wk, gpos, shift), ref)
    assert np.array_equal(run(a[:1], wk, gpos, shift, gemv=True), ref[:1])


def test_w4a8_refuses_group_spread_above_4():
    a, w, gpos, shift = make_case(1, 64, 256, seed=3)
    gpos[1, 5] = gpos[0, 5] + 5
    gpos[0, 5] -= 0
    rc, _ = prepare(w, gpos, 256, 64)
    assert rc == L.IXB_ERR_INVALID


def _u8i4_gpu(a_u8, w_kn, K, N):
    import torch
    lib = L.load()
    gpos = np.zeros((K // 128, N), dtype=np.int8)
    rc, img = prepare(w_kn, gpos, K, N)
    L.check(rc)
    da = _dev(a_u8)
    out = torch.empty((a_u8.shape[0], N), dtype=torch.int32, device="cuda")
    L.check(lib.ixb_u8i4_gemm_i32(C.c_void_p(da.data_ptr()), C.c_void_p(img.data_ptr()), C.c_void_p(out.data_ptr()),
                                  a_u8.shape[0], N, K, None))
    torch.cuda.synchronize()
    return out.cpu().numpy().astype(np.int64)


def test_u8i4_matches_reference_known_answers(golden_dir):
    """The reference's Int4MmulReference tiles (4x8 uint8 x 8x16 int4), zero-padded to K = 128."""
    kat = np.load(golden_dir / "u8i4_kat.npz")
    for i in range(6):
        a = np.zeros((4, 128), dtype=np.uint8)
        a[:, :8] = kat[f"a{i}"]
        w = np.zeros((128, 16), dtype=np.int8)
        w[:8] = O.unpack_int4(kat[f"b{i}_packed"])
        assert np.array_equal(_u8i4_gpu(a, O.pack_int4(w), 128, 16), kat[f"c{i}"])


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (77, 272, 1152), (300, 64, 32768)])
def test_u8i4_gemm_matches_oracle(M, N, K):
    rng = np.random.default_rng(M + K)
    a = rng.integers(0, 256, size=(M, K), dtype=np.uint8)
    if K == 32768:
        a[:] = 255      # the int32 bound: 255 * 8 * K
    w = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    if K == 32768:
        w[:] = -8
    wk = O.pack_int4(w)
    assert np.array_equal(_u8i4_gpu(a, wk, K, N), O.u8i4_i32(a, wk))
