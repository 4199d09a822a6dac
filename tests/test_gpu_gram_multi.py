"""The multi-GPU gram operator (ozk_gram_f64_multi: partial int64 Gram sums
reduced over the ranks) on one GPU: a context of one rank.

With one rank the line maxima of every slice pass are the whole lines'
maxima and the reduced sums are the whole sums, so the pipeline -- the
per-pass line kernels, the symmetric int8 GEMM writing raw int64 sums, the
NCCL all-reduce and the final rounding with the mirror -- must give the
single-GPU gram (ozk_gram_f64) bit for bit.  Also: a NaN raises the flags and
asks for the BF16 recomputation (OZK_FLAG_REDO) instead of writing G, and
shapes without int8 codes are refused (OZK_ERR_UNSUPPORTED)."""

import ctypes

import numpy as np
import pytest
import torch

from ozaki_jax_b200 import _lib as L

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    lib = L.load()
    c = ctypes.c_void_p()
    L.check(lib.ozk_context_create_local(ctypes.byref(c), 1, (ctypes.c_int * 1)(0)))
    yield c
    L.check(lib.ozk_context_destroy(c))


def gram_single(A, n_hi, n_lo):
    lib = L.load()
    N, K = A.shape
    Ad = torch.as_tensor(A).cuda()
    G = torch.empty((K, K), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_bytes = lib.ozk_gram_workspace_bytes(N, K, n_hi, n_lo)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    L.check(lib.ozk_gram_f64(Ad.data_ptr(), K, G.data_ptr(), K, N, K, -1, n_hi, n_lo,
                             ws.data_ptr(), ws_bytes, st.data_ptr(),
                             torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st.item() == 0
    return G.cpu().numpy()


def gram_multi(ctx, A, n_hi, n_lo):
    lib = L.load()
    N, K = A.shape
    Ad = torch.as_tensor(A).cuda()
    G = torch.full((K, K), float("nan"), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    P, I64 = ctypes.c_void_p, ctypes.c_int64
    rc = lib.ozk_gram_f64_multi(ctx, (P * 1)(Ad.data_ptr()), (I64 * 1)(K), (P * 1)(G.data_ptr()),
                                (I64 * 1)(K), N, K, n_hi, n_lo, 0,
                                (P * 1)(torch.cuda.current_stream().cuda_stream),
                                (P * 1)(st.data_ptr()))
    torch.cuda.synchronize()
    return rc, G.cpu().numpy(), int(st.item())


@pytest.mark.parametrize("N,K,n_hi,n_lo,scaled", [(6000, 300, 4, 1, False),
                                                  (20000, 520, 4, 1, True),
                                                  (9000, 256, 3, 1, True),
                                                  (5000, 400, 5, 4, False)])
def test_one_rank_equals_single_gpu_gram(ctx, N, K, n_hi, n_lo, scaled):
    rng = np.random.RandomState(N + K)
    A = rng.randn(N, K)
    if scaled:
        A *= 10.0 ** (-6.0 * np.arange(K) / (K - 1))
    A[:, 7] = 0.0  # a zero line
    rc, G, st = gram_multi(ctx, A, n_hi, n_lo)
    assert rc == 0, L.detail()
    assert st == 0
    assert np.array_equal(G.view(np.int64), gram_single(A, n_hi, n_lo).view(np.int64))
    assert np.array_equal(G, G.T)


def test_nan_flags_and_redo(ctx):
    rng = np.random.RandomState(1)
    A = rng.randn(6000, 300)
    A[123, 45] = np.nan
    rc, G, st = gram_multi(ctx, A, 4, 1)
    assert rc == 0
    assert st & L.OZK_FLAG_NONFINITE and st & L.OZK_FLAG_REDO
    assert np.all(np.isnan(G))  # not written


def test_without_int8_codes_unsupported(ctx):
    A = np.random.RandomState(2).randn(3000, 300)  # rho 18: BF16 slices
    rc, _, _ = gram_multi(ctx, A, 4, 1)
    assert rc == L.OZK_ERR_UNSUPPORTED


@pytest.mark.parametrize("mode", [L.OZK_B_REPLICATED, L.OZK_B_ROOT, L.OZK_B_COLUMNS])
@pytest.mark.parametrize("N,K,M", [(600, 5000, 300), (300, 700, 257)])
def test_one_rank_matmul_multi_equals_single_gpu(ctx, mode, N, K, M):
    """ozk_matmul_f64_multi on a one-rank context, every way of bringing B:
    the single-GPU result (ozk_matmul_f64, fixed-point sums) bit for bit, for
    int8 codes (K = 5000) and BF16 slices (K = 700), blocking and NOWAIT (then
    ozk_context_wait)."""
    lib = L.load()
    rng = np.random.RandomState(N + K + M + mode)
    A, B = rng.randn(N, K), rng.randn(K, M)
    Ad, Bd = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
    ref = torch.empty((N, M), dtype=torch.float64, device="cuda")
    st0 = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    L.check(lib.ozk_matmul_f64(Ad.data_ptr(), K, Bd.data_ptr(), M, ref.data_ptr(), M, N, K, M, -1,
                               4, 1, L.OZK_ACC_FIXED, None, 0, st0.data_ptr(), s))
    P, I64 = ctypes.c_void_p, ctypes.c_int64
    for flags in (0, L.OZK_MULTI_NOWAIT):
        C = torch.full((N, M), float("nan"), dtype=torch.float64, device="cuda")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        L.check(lib.ozk_matmul_f64_multi(
            ctx, (P * 1)(Ad.data_ptr()), (I64 * 1)(K), (P * 1)(Bd.data_ptr()), (I64 * 1)(M),
            (P * 1)(C.data_ptr()), (I64 * 1)(M), N, K, M, 4, 1, mode, flags, (P * 1)(s),
            (P * 1)(st.data_ptr())))
        # the bounded wait of NOWAIT calls (a no-op after a blocking one)
        L.check(lib.ozk_context_wait(ctx, (P * 1)(s)))
        torch.cuda.synchronize()
        assert st.item() == 0 and st0.item() == 0
        assert torch.equal(C.view(torch.int64), ref.view(torch.int64)), (mode, flags)
