"""The rest of the reference's public surface on the device: matmul_numpy,
extract_split_rows/cols (FP64 host-pipeline extraction), accumulate_2sum and
validate_accumulation_2sum, against the oracle (the reference's arithmetic)."""

import numpy as np
import pytest
import torch

import ozaki_jax_b200 as oz
import ozaki_oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_hi,n_lo", [(4, 1), (5, 4), (3, 1), (4, 2)])
def test_accumulate_2sum_bit_exact(n_hi, n_lo):
    rng = np.random.RandomState(n_hi * 10 + n_lo)
    A, B = rng.randn(40, 300) * np.exp(rng.randn(40, 1)), rng.randn(300, 33)
    SA, eA, SB, eB, _ = O.extract_ondevice(A, B, n_hi, n_lo)
    pairs, _, _ = O.ondevice_pairs(n_hi, n_lo)
    P = O.slice_products(SA, SB, pairs)
    col, row, bgs = O.accumulation_scales(eA, eB, n_hi, n_lo)
    ref_hi, ref_lo = O.accumulate_2sum(P, col, row, bgs)
    hi, lo = oz.accumulate_2sum(P, col, row, bgs)
    assert isinstance(hi, np.ndarray) and hi.dtype == np.float32
    assert same_bits(hi, ref_hi) and same_bits(lo, ref_lo)
    dhi, dlo = oz.accumulate_2sum(torch.as_tensor(P).cuda(), torch.as_tensor(col).cuda(),
                                  torch.as_tensor(row).cuda(), bgs, backend="pallas")
    assert dhi.is_cuda and same_bits(dhi.cpu().numpy(), ref_hi)


def test_accumulate_2sum_arguments():
    with pytest.raises(ValueError, match="Unknown backend='tpu'; expected 'auto', 'jax', or 'pallas'."):
        oz.accumulate_2sum(np.zeros((1, 2, 2), np.float32), np.ones((1, 2), np.float32),
                           np.ones((1, 2), np.float32), ((1,),), backend="tpu")
    with pytest.raises(ValueError):
        oz.accumulate_2sum(np.zeros((2, 2, 2), np.float32), np.ones((2, 2), np.float32),
                           np.ones((1, 2), np.float32), ((1,),))


def test_validate_accumulation_2sum():
    r = oz.validate_accumulation_2sum()
    assert r["match"] and r["N"] == r["M"] == r["K"] == 128
    assert r["max_rel_error"] < 1e-9 and r["baseline_error"] < 1e-14


@pytest.mark.parametrize("shape", [(37, 100), (64, 2000), (5, 1)])
def test_extract_split_rows_cols_bit_exact(shape):
    rng = np.random.RandomState(sum(shape))
    X = rng.randn(*shape) * np.exp(3 * rng.randn(*shape))
    rho = O.compute_rho_f64(shape[1])
    S, E = oz.extract_split_rows(X, rho, 8)
    RS, RE = O.extract_rows_f64(X, rho, 8)
    assert len(S) == 8 and S[0].dtype == np.float32 and E[0].dtype == np.float64
    assert all(same_bits(a, b) for a, b in zip(S, RS))
    assert all(np.array_equal(a, b) for a, b in zip(E, RE))
    rho_c = O.compute_rho_f64(shape[0])
    S, E = oz.extract_split_cols(X, rho_c, 6)
    RS, RE = O.extract_cols_f64(X, rho_c, 6)
    assert all(same_bits(a, b) for a, b in zip(S, RS))
    assert all(np.array_equal(a, b) for a, b in zip(E, RE))


def test_matmul_numpy_both_pipelines():
    rng = np.random.RandomState(3)
    A, B = rng.randn(96, 700), rng.randn(700, 80)
    E = O.exact_product(A, B)
    for precision in ("high", "max"):
        n_hi, n_lo = O.resolve_precision(precision)
        C = oz.matmul_numpy(A, B, pipeline="ondevice", precision=precision)
        R = O.ondevice_numpy(A, B, n_hi, n_lo)
        assert isinstance(C, np.ndarray) and C.shape == (96, 80)
        assert O.rel_err(C, E) <= max(1.5 * O.rel_err(R, E), 32 * 2.0 ** -52)
    C = oz.matmul_numpy(A, B, n_slices=8, pipeline="host")
    assert O.rel_err(C, E) <= max(1.5 * O.rel_err(O.host_numpy(A, B, 8), E), 32 * 2.0 ** -52)
    with pytest.raises(ValueError, match="Unknown pipeline='gpu'"):
        oz.matmul_numpy(A, B, pipeline="gpu")
