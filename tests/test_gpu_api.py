"""The drop-in API on the device: the reference's CI pins
(benchmarks/ci_cpu_validate.py, ci_gram_validate.py, ci_solve_validate.py),
type policy, preflight behaviour and edge shapes."""

import numpy as np
import pytest
import torch

import ozaki_jax_b200 as oz
import ozaki_oracle as O

pytestmark = pytest.mark.gpu


def rel(a, r):
    a = a.cpu().numpy() if isinstance(a, torch.Tensor) else a
    return O.rel_err(a, r)


def test_ci_cpu_validate_pins():
    rng = np.random.RandomState(0)
    A, B = rng.randn(64, 64), rng.randn(64, 64)
    R = A @ B
    for acc in ("host", "ondevice", "fused", "bf16_interleaved"):
        C = oz.matmul(A, B, pipeline="ondevice", accumulation=acc)
        assert isinstance(C, np.ndarray) and C.shape == (64, 64) and C.dtype == np.float64
        assert rel(C, R) <= 1e-9, acc
    cf = oz.matmul(A, B, pipeline="ondevice", accumulation="fused")
    cd = oz.matmul(A, B, pipeline="ondevice", accumulation="ondevice")
    assert rel(cf, cd) <= 1e-9
    for acc in ("host", "fused"):
        assert rel(oz.matmul(A, B, pipeline="ondevice", accumulation=acc, precision="max"),
                   R) <= 1e-14, acc
    assert rel(oz.matmul(A, B, pipeline="ondevice", precision="medium"), R) <= 1e-6
    assert rel(oz.matmul(A, B, pipeline="ondevice", precision=(4, 2)), R) <= 1e-9


def test_device_in_device_out():
    rng = np.random.RandomState(0)
    A, B = rng.randn(64, 64), rng.randn(64, 64)
    At, Bt = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
    for acc in ("fused", "ondevice", "host"):
        C = oz.matmul(At, Bt, pipeline="ondevice", accumulation=acc)
        assert isinstance(C, torch.Tensor) and C.is_cuda and C.dtype == torch.float64
        assert rel(C, A @ B) <= 1e-9
    # float32 / non-contiguous device inputs are converted like jnp.asarray(f64)
    C = oz.matmul(At.T.float(), Bt, pipeline="ondevice")
    assert rel(C, A.T.astype(np.float32).astype(np.float64) @ B) <= 1e-9


def test_nonfinite_raise_and_fallback(golden):
    _, meta = golden
    A = np.full((4, 4), np.nan)
    with pytest.raises(ValueError) as ei:
        oz.matmul(A, np.ones((4, 4)), pipeline="ondevice")
    assert str(ei.value) == meta["messages"]["ondevice_nan"]
    with pytest.raises(ValueError) as ei:
        oz.matmul(np.ones((4, 4)), np.full((4, 4), np.inf), pipeline="ondevice")
    assert str(ei.value) == meta["messages"]["ondevice_inf"]
    A = np.ones((3, 5))
    A[1, 2] = np.inf
    B = np.arange(10.0).reshape(5, 2)
    C = oz.matmul(A, B, pipeline="ondevice", safe_mode="fallback")
    assert np.array_equal(np.isnan(C), np.isnan(A @ B))
    big = np.ones((2, 3))
    big[0, 0] = 1e300
    with pytest.raises(ValueError, match="FP32 range"):
        oz.matmul(big, np.ones((3, 2)), pipeline="ondevice")


@pytest.mark.parametrize("N,K,M", [(1, 128, 1), (128, 1, 128), (129, 257, 65), (300, 70, 5),
                                   (1, 1, 1), (7, 3000, 260)])
def test_edge_shapes(N, K, M):
    rng = np.random.RandomState(N * 7 + K * 3 + M)
    A, B = rng.randn(N, K), rng.randn(K, M)
    E = O.exact_product(A, B)
    C = oz.matmul(A, B, pipeline="ondevice")
    ref = O.ondevice_numpy(A, B, 4, 1)
    assert C.shape == (N, M)
    assert O.rel_err(C, E) <= max(1.5 * O.rel_err(ref, E), 32 * 2.0 ** -52)


def test_empty_shapes():
    assert oz.matmul(np.ones((0, 5)), np.ones((5, 3)), pipeline="ondevice").shape == (0, 3)
    assert oz.matmul(np.ones((4, 5)), np.ones((5, 0)), pipeline="ondevice").shape == (4, 0)
    with pytest.raises(ValueError):
        oz.matmul(np.ones((4, 0)), np.ones((0, 3)), pipeline="ondevice")


def test_gram_pins(golden):
    arrays, _ = golden
    rng = np.random.RandomState(42)
    A = rng.randn(128, 128)
    G_ref = A.T @ A
    G = oz.gram(A, mode="ozaki", precision="high")
    assert isinstance(G, np.ndarray) and G.shape == (128, 128)
    assert rel(G, G_ref) <= 1e-9
    assert np.array_equal(G, G.T)
    assert rel(oz.gram(A, mode="ozaki", precision="medium"), G_ref) <= 1e-5
    assert rel(oz.gram(A, mode="ozaki", accumulation="fused"), G_ref) <= 1e-9
    assert rel(oz.gram(A), G_ref) <= 1e-14
    Gt = oz.gram(torch.as_tensor(A).cuda(), mode="ozaki")
    assert isinstance(Gt, torch.Tensor)
    # golden: column-scaled tall matrix, within 1.5x of the reference's error
    GA = arrays["gram/A"]
    E = O.exact_product(GA.T, GA)
    for pname in ("high", "medium"):
        G = oz.gram(GA, mode="ozaki", precision=pname)
        ref = arrays[f"gram/{pname}/bf16_interleaved"]
        assert O.rel_err(G, E) <= 1.5 * O.rel_err(ref, E), pname
        assert np.array_equal(G, G.T)


def test_residual_pins(golden):
    arrays, _ = golden
    A, x, b = arrays["residual/A"], arrays["residual/x"], arrays["residual/b"]
    Ax = O.exact_product(A, x)
    for pname in ("high", "medium"):
        r = oz.residual(A, x, b, mode="ozaki", precision=pname)
        ref = arrays[f"residual/{pname}/bf16_interleaved"]
        err = np.linalg.norm(r - (b - Ax)) / np.linalg.norm(b - Ax)
        err_ref = np.linalg.norm(ref - (b - Ax)) / np.linalg.norm(b - Ax)
        assert err <= 1.5 * err_ref + 1e-15, pname
    xv, bv = arrays["residual/xv"], arrays["residual/bv"]
    rv = oz.residual(A, xv, bv, mode="ozaki")
    assert rv.shape == (64,)
    assert O.rel_err(rv, arrays["residual/high/vec"]) <= 1e-6
    rng = np.random.RandomState(1)
    A2, x2, b2 = rng.randn(64, 128), rng.randn(128), rng.randn(64)
    assert rel(oz.residual(A2, x2, b2, mode="ozaki"), b2 - A2 @ x2) <= 1e-9
    assert rel(oz.residual(A2, x2, b2), b2 - A2 @ x2) <= 1e-14
