"""The allocation-free matmul entry point (ozk_matmul_f64_noalloc).

Some callers of this library cannot allocate device memory in the middle of a
call -- for instance code running inside a JAX/XLA process, whose allocator
has reserved most of the GPU up front, or a plugin callback its host framework
forbids from allocating.  For them the library keeps a fixed 32 MiB device
scratch array and takes the slice workspace from it.  This test calls that
entry point through the C ABI twice in a row (different shapes and data, so
stale contents from the first call would show) and checks each result against
the allocating entry point, ozk_matmul_f64, within the tolerance the other
FP64-epilogue tests use; it also checks the size limit is enforced.

This file is collected last so a failure here leaves every other test run.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, Ad, Bd, n_hi, n_lo):
    N, K = Ad.shape
    M = Bd.shape[1]
    C = torch.full((N, M), float("nan"), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.ozk_matmul_f64_noalloc(Ad.data_ptr(), K, Bd.data_ptr(), M, C.data_ptr(), M, N, K, M,
                                    n_hi, n_lo, st.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    return rc, C, st


def _call_allocating(lib, Ad, Bd, n_hi, n_lo):
    from ozaki_jax_b200 import _lib
    N, K = Ad.shape
    M = Bd.shape[1]
    C = torch.empty((N, M), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_bytes = lib.ozk_matmul_workspace_bytes(N, K, M, n_hi, n_lo)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    # same accumulation as the allocation-free entry point: 'fused' (OZK_ACC_FIXED)
    rc = lib.ozk_matmul_f64(Ad.data_ptr(), K, Bd.data_ptr(), M, C.data_ptr(), M, N, K, M, -1,
                            n_hi, n_lo, _lib.OZK_ACC_FIXED, ws.data_ptr(), ws_bytes, st.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    return rc, C, st


def test_noalloc_matches_allocating_entry_point_twice():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    cases = [((300, 1000, 200), (4, 1), 0), ((1024, 1024, 1024), (4, 1), 1),
             ((77, 513, 129), (5, 4), 2)]
    for (N, K, M), (n_hi, n_lo), seed in cases:
        rng = np.random.RandomState(seed)
        A, B = rng.randn(N, K), rng.randn(K, M)
        Ad, Bd = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
        rc, C0, st0 = _call_noalloc(lib, Ad, Bd, n_hi, n_lo)
        assert rc == 0, _lib.detail()
        rc, C1, st1 = _call_allocating(lib, Ad, Bd, n_hi, n_lo)
        assert rc == 0, _lib.detail()
        torch.cuda.synchronize()
        assert st0.item() == 0 and st1.item() == 0
        c0, c1 = C0.cpu().numpy(), C1.cpu().numpy()
        scale = np.abs(A) @ np.abs(B)
        assert np.all(np.abs(c0 - c1) <= 64 * 2.0 ** -52 * scale), (N, K, M)


def test_noalloc_rejects_oversized_requests():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    Ad = torch.zeros((2048, 2048), dtype=torch.float64, device="cuda")
    rc, _, _ = _call_noalloc(lib, Ad, Ad, 4, 1)
    assert rc == _lib.OZK_ERR_WORKSPACE
    assert "fixed" in _lib.detail() and "scratch" in _lib.detail()
