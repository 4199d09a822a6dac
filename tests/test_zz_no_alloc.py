"""The allocation-free matmul entry point (ozk_matmul_f64_noalloc).

Some callers of this library cannot allocate device memory in the middle of a
call -- for instance code running inside a JAX/XLA process, whose allocator
has reserved most of the GPU up front, or a plugin callback its host framework
forbids from allocating.  For them the library keeps a fixed 32 MiB device
scratch array and takes the slice workspace from it.

This test calls that entry point through the C ABI on several cases in a row
(different shapes and data, so stale contents from an earlier call would
show) and checks each result against the allocating entry point,
ozk_matmul_f64 with the same accumulation (OZK_ACC_FIXED).  Both compute
exact fixed-point sums of the same exact slice products, so the results must
be bit-identical even though different GEMM tiles run (the allocation-free
call has no room for the wide tiles' state scratch).  One case is also held
to the CPU oracle: element by element against the reference's FP64 pipeline
within the fixed-point resolution, and normwise no worse than 1.5x the
reference's own error against the exact product.  The size limit is checked
too.

This file is collected last so a failure here leaves every other test run.
"""

import numpy as np
import pytest
import torch

import ozaki_oracle as O

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


def test_noalloc_bit_identical_to_allocating_entry_point():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    cases = [((300, 1000, 200), (4, 1), 0), ((1024, 1024, 1024), (4, 1), 1),
             ((77, 513, 129), (5, 4), 2), ((300, 1000, 200), (4, 1), 3),
             ((512, 5000, 8), (4, 1), 4)]
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
        assert np.array_equal(c0, c1), ((N, K, M), float(np.max(np.abs(c0 - c1))))
        if seed == 0:
            # the CPU oracle: the reference's FP64 pipeline within the fixed-point
            # resolution, and the reference's own error bound against the exact product
            ref = O.ondevice_numpy(A, B, n_hi, n_lo)
            rmax = np.max(np.abs(A), axis=1)[:, None]
            cmax = np.max(np.abs(B), axis=0)[None, :]
            n_pairs = n_hi * n_hi + 2 * n_hi * n_lo
            bound = n_pairs * 2.0 ** -48 * rmax * cmax + 64 * 2.0 ** -52 * (np.abs(A) @ np.abs(B))
            assert np.all(np.abs(c0 - ref) <= bound)
            E = O.exact_product(A, B)
            assert O.rel_err(c0, E) <= max(1.5 * O.rel_err(ref, E), 32 * 2.0 ** -52)


def test_noalloc_rejects_oversized_requests():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    Ad = torch.zeros((2048, 2048), dtype=torch.float64, device="cuda")
    rc, _, _ = _call_noalloc(lib, Ad, Ad, 4, 1)
    assert rc == _lib.OZK_ERR_WORKSPACE
    assert "fixed" in _lib.detail() and "scratch" in _lib.detail()
