"""ozk_matmul_f64_hostbuf (host arrays in and out, copies overlapped with the
compute in row blocks) against ozk_matmul_f64 on device arrays: the blocking
must not change a single bit, for every accumulation mode, ragged last
blocks, strided host arrays, pinned and pageable host memory."""

import ctypes

import numpy as np
import pytest
import torch

import ozaki_jax_b200 as oz
from ozaki_jax_b200 import _lib as L

pytestmark = pytest.mark.gpu

MODES = [L.OZK_ACC_FIXED, L.OZK_ACC_F64, L.OZK_ACC_PRODUCTS]


def device_result(A, B, n_hi, n_lo, mode):
    lib = L.load()
    Ad, Bd = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
    N, K = A.shape
    M = B.shape[1]
    C = torch.empty((N, M), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_bytes = lib.ozk_matmul_workspace_bytes(N, K, M, n_hi, n_lo)
    if mode == L.OZK_ACC_PRODUCTS:
        ws_bytes += (n_hi * n_hi + 2 * n_hi * n_lo) * N * M * 4 + 256
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    L.check(lib.ozk_matmul_f64(Ad.data_ptr(), K, Bd.data_ptr(), M, C.data_ptr(), M, N, K, M, -1,
                               n_hi, n_lo, mode, ws.data_ptr(), ws_bytes, st.data_ptr(),
                               torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st.item() == 0
    return C.cpu().numpy()


def hostbuf(A, B, n_hi, n_lo, mode, block_rows=0, C=None, with_ws=True):
    """A, B, C may be strided row-major views (unit column stride)."""
    lib = L.load()
    N, K = A.shape
    M = B.shape[1]
    if C is None:
        C = np.full((N, M), np.nan)
    ws_bytes = lib.ozk_matmul_hostbuf_workspace_bytes(N, K, M, n_hi, n_lo, mode, block_rows)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda") if with_ws else None
    flags = ctypes.c_int32(-1)
    L.check(lib.ozk_matmul_f64_hostbuf(
        A.ctypes.data, A.strides[0] // 8, B.ctypes.data, B.strides[0] // 8, C.ctypes.data,
        C.strides[0] // 8, N, K, M, -1, n_hi, n_lo, mode, block_rows,
        ws.data_ptr() if with_ws else None, ws_bytes if with_ws else 0, ctypes.byref(flags),
        torch.cuda.current_stream().cuda_stream))
    return C, flags.value


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("block_rows", [0, 256, 384])
def test_blocked_equals_device_pipeline(mode, block_rows):
    rng = np.random.RandomState(3)
    A = rng.randn(1100, 300) * np.exp(rng.randn(1100, 1))
    B = rng.randn(300, 700) * np.exp(rng.randn(1, 700))
    C, flags = hostbuf(A, B, 4, 1, mode, block_rows)
    assert flags == 0
    R = device_result(A, B, 4, 1, mode)
    assert np.array_equal(C.view(np.int64), R.view(np.int64))


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("K", [300, 4224])  # BF16 slices; int8 codes (rho 19)
def test_uneven_row_blocks(mode, K):
    # N = 1100 -> row blocks of 768 and 332 (a short last block): every block's
    # extraction and GEMM give exactly the rows of the whole product
    rng = np.random.RandomState(11)
    A = rng.randn(1100, K) * np.exp(rng.randn(1100, 1))
    B = rng.randn(K, 1300) * np.exp(rng.randn(1, 1300))
    C, flags = hostbuf(A, B, 4, 1, mode)
    assert flags == 0
    R = device_result(A, B, 4, 1, mode)
    assert np.array_equal(C.view(np.int64), R.view(np.int64))


@pytest.mark.parametrize("mode", [L.OZK_ACC_FIXED, L.OZK_ACC_F64])
def test_automatic_blocks_full_height(mode):
    # N = 8192 -> automatic blocks of 1024 rows, as in the 8192^3 benchmark
    # (int8 codes at K = 4224): still the whole product's rows
    rng = np.random.RandomState(12)
    A = rng.randn(8192, 4224) * np.exp(rng.randn(8192, 1))
    B = rng.randn(4224, 300) * np.exp(rng.randn(1, 300))
    C, flags = hostbuf(A, B, 4, 1, mode)
    assert flags == 0
    R = device_result(A, B, 4, 1, mode)
    assert np.array_equal(C.view(np.int64), R.view(np.int64))


def test_strided_and_pinned_host_arrays():
    rng = np.random.RandomState(4)
    Abig = rng.randn(700, 260)
    Bbig = rng.randn(200, 530)
    A, B = Abig[:, 10:210], Bbig[:, 3:515]  # lda 260, ldb 530
    Cbig = np.full((700, 600), -7.0)
    C = Cbig[:, 50:562]
    out, flags = hostbuf(A, B, 4, 1, L.OZK_ACC_FIXED, block_rows=256, C=C)
    assert flags == 0
    R = device_result(np.ascontiguousarray(A), np.ascontiguousarray(B), 4, 1, L.OZK_ACC_FIXED)
    assert np.array_equal(C.view(np.int64), R.view(np.int64))
    # the columns outside C's window are untouched
    assert np.all(Cbig[:, :50] == -7.0) and np.all(Cbig[:, 562:] == -7.0)
    # pinned copies of the same data give the same bits
    pA = torch.empty(A.shape, dtype=torch.float64, pin_memory=True).numpy()
    pB = torch.empty(B.shape, dtype=torch.float64, pin_memory=True).numpy()
    pC = torch.empty((700, 512), dtype=torch.float64, pin_memory=True).numpy()
    pA[...] = A
    pB[...] = B
    hostbuf(pA, pB, 4, 1, L.OZK_ACC_FIXED, C=pC)
    assert np.array_equal(pC.view(np.int64), R.view(np.int64))


def test_pool_workspace_and_presets():
    rng = np.random.RandomState(5)
    A, B = rng.randn(300, 1000), rng.randn(1000, 260)
    for n_hi, n_lo in ((3, 1), (5, 4)):
        C, flags = hostbuf(A, B, n_hi, n_lo, L.OZK_ACC_FIXED, with_ws=False)
        assert flags == 0
        R = device_result(A, B, n_hi, n_lo, L.OZK_ACC_FIXED)
        assert np.array_equal(C.view(np.int64), R.view(np.int64))


def test_nonfinite_flag_reported_on_host():
    A = np.ones((64, 64))
    A[5, 7] = np.nan
    _, flags = hostbuf(A, np.ones((64, 64)), 4, 1, L.OZK_ACC_FIXED)
    assert flags & L.OZK_FLAG_NONFINITE


def test_public_api_numpy_path_uses_hostbuf_result():
    rng = np.random.RandomState(6)
    A, B = rng.randn(1500, 400), rng.randn(400, 900)
    C = oz.matmul(A, B, pipeline="ondevice")
    assert isinstance(C, np.ndarray) and C.dtype == np.float64 and C.shape == (1500, 900)
    R = device_result(A, B, 4, 1, L.OZK_ACC_FIXED)
    assert np.array_equal(C.view(np.int64), R.view(np.int64))
    Cd = oz.matmul(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), pipeline="ondevice")
    assert np.array_equal(Cd.cpu().numpy().view(np.int64), C.view(np.int64))


def test_staged_copies_round_trip():
    """ozk_memcpy_staged between pageable host memory and the device: sizes
    below one row, across several staging slots and with ragged tails come
    back byte for byte; page-locked memory takes the direct path."""
    lib = L.load()
    s = torch.cuda.current_stream().cuda_stream
    rng = np.random.RandomState(9)
    for n in (1, 8, (1 << 20) + 3, (100 << 20) + 5):
        src = rng.randint(0, 256, size=n, dtype=np.uint8)
        dev = torch.empty(n, dtype=torch.uint8, device="cuda")
        L.check(lib.ozk_memcpy_staged(dev.data_ptr(), src.ctypes.data, n, s))
        assert np.array_equal(dev.cpu().numpy(), src), n
        dev.add_(1)
        back = np.zeros(n, dtype=np.uint8)
        L.check(lib.ozk_memcpy_staged(back.ctypes.data, dev.data_ptr(), n, s))
        assert np.array_equal(back, (src + 1).astype(np.uint8)), n
    pinned = torch.empty(1 << 20, dtype=torch.uint8, pin_memory=True)
    pinned.numpy()[...] = 7
    dev = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    L.check(lib.ozk_memcpy_staged(dev.data_ptr(), pinned.data_ptr(), 1 << 20, s))
    assert int(dev.sum().item()) == 7 << 20


def test_pageable_large_operands_staged_in_many_chunks():
    """Pageable A, B and C several times the staging slots (32 MiB), with a
    strided C: bit-identical to the device pipeline, untouched outside C."""
    rng = np.random.RandomState(13)
    A = rng.randn(4096, 1500)
    B = rng.randn(1500, 4096)
    Cbig = np.full((4096, 4100), -3.0)
    C = Cbig[:, 2:4098]
    out, flags = hostbuf(A, B, 4, 1, L.OZK_ACC_FIXED, C=C)
    assert flags == 0
    R = device_result(A, B, 4, 1, L.OZK_ACC_FIXED)
    assert np.array_equal(C.view(np.int64), R.view(np.int64))
    assert np.all(Cbig[:, :2] == -3.0) and np.all(Cbig[:, 4098:] == -3.0)
