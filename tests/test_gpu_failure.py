"""Failure detection without a GPU fault: every device-side wait is bounded.

A self-test kernel waits on an mbarrier that nothing arrives at; the wait must
give up after its budget, report OZK_FLAG_TIMEOUT, and leave the context
usable (a matmul right after it still succeeds)."""

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ok = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _lib.check(lib.ozk_selftest_timeout(20, status.data_ptr(), ok.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert ok.item() == 0
    assert status.item() & _lib.OZK_FLAG_TIMEOUT
    assert dt < 5.0
    assert lib.ozk_check_status(status.data_ptr(), torch.cuda.current_stream().cuda_stream) == \
        _lib.OZK_ERR_TIMEOUT
    # the context is still healthy
    import ozaki_jax_b200 as oz
    rng = np.random.RandomState(0)
    A, B = rng.randn(64, 64), rng.randn(64, 64)
    C = oz.matmul(A, B, pipeline="ondevice")
    assert np.linalg.norm(C - A @ B) / np.linalg.norm(A @ B) < 1e-9


def test_timeout_flag_maps_to_error():
    from ozaki_jax_b200 import _lib
    from ozaki_jax_b200.matmul import _read_status
    st = torch.tensor([_lib.OZK_FLAG_TIMEOUT], dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.OzakiError):
        _read_status(st)
