"""matmul(pipeline='host') on the device: FP64 extraction bit-identical to the
oracle of ozaki_jax/extract.py:21-103, triangular pairs, FP64 accumulation;
the reference's CI pins and the 256 x 256, n_slices=8 CPU-plumbing case."""

import numpy as np
import pytest
import torch

import ozaki_jax_b200 as oz
import ozaki_oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu


def dev_extract64(X, rho, n, axis):
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    Xd = torch.as_tensor(np.ascontiguousarray(X)).cuda()
    if axis == 1:
        lines, K = X.shape
    else:
        K, lines = X.shape
    k_pad = (K + 63) // 64 * 64
    S = torch.empty((n, lines, k_pad), dtype=torch.int16, device="cuda")
    E = torch.empty((n, lines), dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    fn = lib.ozk_extract_rows_host_f64 if axis == 1 else lib.ozk_extract_cols_host_f64
    dims = (lines, K) if axis == 1 else (K, lines)
    _lib.check(fn(Xd.data_ptr(), X.shape[1], *dims, rho, n, S.data_ptr(), k_pad, E.data_ptr(),
                  st.data_ptr(), torch.cuda.current_stream().cuda_stream))
    bits = S.cpu().numpy().view(np.uint16)[:, :, :K].astype(np.uint32) << 16
    return bits.view(np.float32), E.cpu().numpy(), int(st.item())


@pytest.mark.parametrize("shape,seed,wide", [((64, 64), 0, False), ((37, 300), 1, True),
                                             ((5, 5000), 2, False)])
def test_fp64_extraction_matches_oracle(shape, seed, wide):
    rng = np.random.RandomState(seed)
    X = rng.randn(*shape)
    if wide:
        X = (rng.rand(*shape) - 0.5) * np.exp(10 * rng.randn(*shape))
    rho = O.compute_rho_f64(shape[1])
    s, e, st = dev_extract64(X, rho, 8, axis=1)
    rs, re_ = O.extract_rows_f64(X, rho, 8)
    assert st == 0
    assert same_bits(s, np.stack(rs))
    assert np.array_equal(e, np.stack(re_).astype(np.int32))
    rho = O.compute_rho_f64(shape[0])
    s, e, st = dev_extract64(X, rho, 8, axis=0)
    cs, ce = O.extract_cols_f64(X, rho, 8)
    assert same_bits(s, np.stack(cs).transpose(0, 2, 1))
    assert np.array_equal(e, np.stack(ce).astype(np.int32))


def test_host_pipeline_goldens(golden):
    arrays, _ = golden
    for name in ("n64_s0", "rect_37x100x23", "zeros_24x48x16", "wide_phi10_40x96x32",
                 "log2_edges_12x20x10", "vec_1x128x1", "outer_48x1x40"):
        A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
        E = O.exact_product(A, B)
        C = oz.matmul(A, B)
        ref = arrays[f"{name}/host8"]
        assert O.rel_err(C, E) <= max(1.5 * O.rel_err(ref, E), 32 * 2.0 ** -52), name


def test_host_ci_pins():
    rng = np.random.RandomState(0)
    A, B = rng.randn(64, 64), rng.randn(64, 64)
    assert O.rel_err(oz.matmul(A, B, pipeline="host"), A @ B) <= 1e-14
    A_bad, B_bad = rng.randn(2, 10_000), rng.randn(10_000, 2)
    C = oz.matmul(A_bad, B_bad, pipeline="host", safe_mode="fallback")
    assert O.rel_err(C, A_bad @ B_bad) <= 1e-14
    with pytest.raises(ValueError, match="insufficient slice budget"):
        oz.matmul(A_bad, B_bad, pipeline="host")
    with pytest.raises(ValueError, match="n_slices must be >= 1"):
        oz.matmul(A, B, n_slices=0)


def test_config1_256_host_pipeline():
    """The plumbing case: 256x256 N(0,1) seed 0, n_slices=8 -> ~5.6e-16."""
    rng = np.random.RandomState(0)
    A, B = rng.randn(256, 256), rng.randn(256, 256)
    E = O.exact_product(A, B)
    C = oz.matmul(A, B, n_slices=8, safe_mode="raise")
    ref = O.host_numpy(A, B, 8)
    assert O.rel_err(C, E) <= max(1.5 * O.rel_err(ref, E), 32 * 2.0 ** -52)
    assert O.rel_err(C, E) < 2e-15
