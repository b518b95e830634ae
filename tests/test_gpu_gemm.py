"""int8 GEMM + SRS and raw int32 GEMM on a B200 through the C ABI, against the oracle (numpy
int64), bit-exact: square sizes, YOLOv8n convs as im2col GEMMs, ragged M and N tails, K tails."""
import ctypes as C

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _operands(M, N, K, seed, dist="uniform"):
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        a = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
        b = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    else:
        a = np.clip(np.rint(rng.normal(0, 32, size=(M, K))), -127, 127).astype(np.int8)
        b = np.clip(np.rint(rng.normal(0, 32, size=(N, K))), -127, 127).astype(np.int8)
    bias = rng.integers(-(1 << 20), 1 << 20, size=N, dtype=np.int32)
    return a, b, bias


def run_srs(a, b, bias, shift):
    import torch
    lib = L.load()
    M, K = a.shape
    N = b.shape[0]
    da, db, dbias = _dev(a), _dev(b), _dev(bias)
    out = torch.empty((M, N), dtype=torch.int8, device="cuda")
    L.check(lib.ixb_i8gemm_srs(C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr()), C.c_void_p(dbias.data_ptr()),
                               C.c_void_p(out.data_ptr()), M, N, K, shift, None))
    torch.cuda.synchronize()
    L.check(lib.ixb_device_error(C.byref(C.c_int())))
    return out.cpu().numpy()


def run_i32(a, b):
    import torch
    lib = L.load()
    M, K = a.shape
    N = b.shape[0]
    da, db = _dev(a), _dev(b)
    out = torch.empty((M, N), dtype=torch.int32, device="cuda")
    L.check(lib.ixb_i8gemm_i32(C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr()), C.c_void_p(out.data_ptr()),
                               M, N, K, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("M,N,K,shift,dist", [
    (256, 256, 256, 3, "uniform"), (1024, 1024, 1024, 12, "normal"), (512, 768, 384, 8, "uniform"),
    (1000, 48, 144, 7, "uniform"), (129, 16, 16, 0, "normal"), (300, 272, 1040, 10, "normal"),
    (2 * 160 * 160, 32, 288, 9, "normal"), (2 * 80 * 80, 64, 576, 10, "uniform"), (2 * 20 * 20, 256, 2304, 11, "normal"),
])
def test_i8gemm_srs_matches_oracle(M, N, K, shift, dist):
    a, b, bias = _operands(M, N, K, seed=M + N + K, dist=dist)
    got = run_srs(a, b, bias, shift)
    assert np.array_equal(got, O.i8gemm_srs(a, b, bias, shift))


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (4096, 512, 4096), (333, 400, 208), (128, 512, 8192)])
def test_i8gemm_i32_is_exact(M, N, K):
    a, b, _ = _operands(M, N, K, seed=7 + K)
    got = run_i32(a, b)
    ref = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(got.astype(np.int64), ref)


def test_i8gemm_extremes_saturate_and_round_to_even():
    """All -127 / 127 operands (largest |acc|), and accumulators landing on exact halves."""
    M, N, K = 256, 64, 4096
    a = np.full((M, K), 127, dtype=np.int8)
    a[::2] = -127
    b = np.full((N, K), 127, dtype=np.int8)
    bias = np.zeros(N, dtype=np.int32)
    assert np.array_equal(run_srs(a, b, bias, 12), O.i8gemm_srs(a, b, bias, 12))
    a = np.zeros((M, 32), dtype=np.int8)
    a[:, 0] = np.arange(M) - 128
    b = np.zeros((N, 32), dtype=np.int8)
    b[:, 0] = 1
    bias = (np.arange(N, dtype=np.int32) * 3) - 90
    assert np.array_equal(run_srs(a, b, bias, 2), O.i8gemm_srs(a, b, bias, 2))
    # a bias that pushes the sum past int32 still saturates to the right int8
    a = np.full((M, 64), 127, dtype=np.int8)
    b = np.full((N, 64), 127, dtype=np.int8)
    bias = np.full(N, 2**31 - 1000, dtype=np.int32)
    bias[1::2] = -(2**31)
    assert np.array_equal(run_srs(a, b, bias, 23), O.i8gemm_srs(a, b, bias, 23))


@pytest.mark.parametrize("sms", ["4", "16"])
def test_i8gemm_many_tiles_per_cta(sms, monkeypatch):
    """A planner SM count below the tile count: each CTA runs several tiles through its TMEM
    accumulators (the persistent loop's accumulator rotation and phases), SRS and int32 forms."""
    monkeypatch.setenv("IXB_SM_COUNT", sms)
    M, N, K = 2048, 1024, 512
    a, b, bias = _operands(M, N, K, seed=31)
    assert np.array_equal(run_srs(a, b, bias, 9), O.i8gemm_srs(a, b, bias, 9))
    assert np.array_equal(run_i32(a, b).astype(np.int64), a.astype(np.int64) @ b.astype(np.int64).T)
