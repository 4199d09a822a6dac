"""K1 parity: device slices and exponents are bit-identical to the reference
(golden vectors) and to the oracle, through the C ABI."""

import numpy as np
import pytest
import torch

import ozaki_oracle as O
from conftest import bf16_bits_to_f32, same_bits

pytestmark = pytest.mark.gpu

CASES = ["n64_s0", "rect_37x100x23", "zeros_24x48x16", "wide_phi10_40x96x32",
         "k1040_8x1040x8", "scales_16x32x12", "log2_edges_12x20x10", "vec_1x128x1",
         "outer_48x1x40"]


def dev_extract(X, rho, n_hi, n_lo, axis):
    from ozaki_jax_b200.extract import extract_device
    Xd = torch.as_tensor(np.ascontiguousarray(X, dtype=np.float64)).cuda()
    S, k_pad, E, st = extract_device(Xd, rho, n_hi, n_lo, axis)
    K = X.shape[1] if axis == 1 else X.shape[0]
    bits = S.cpu().numpy().view(np.uint16)
    assert np.all(bits[:, :, K:] == 0), "K padding must be zero"
    return bits[:, :, :K], E.cpu().numpy(), int(st.item())


@pytest.mark.parametrize("name", CASES)
def test_slices_match_reference_goldens(golden, name):
    arrays, meta = golden
    A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
    rho = meta["cases"][name]["rho"]
    sa, ea, _ = dev_extract(A, rho, 5, 5, axis=1)
    sb, eb, _ = dev_extract(B, rho, 5, 5, axis=0)
    ref_a = np.concatenate([arrays[f"{name}/A_hi/slices"], arrays[f"{name}/A_lo/slices"]])
    ref_b = np.concatenate([arrays[f"{name}/B_hi/slices"], arrays[f"{name}/B_lo/slices"]])
    assert same_bits(bf16_bits_to_f32(sa), bf16_bits_to_f32(ref_a))
    assert same_bits(bf16_bits_to_f32(sb), bf16_bits_to_f32(ref_b).transpose(0, 2, 1))
    ref_ea = np.concatenate([arrays[f"{name}/A_hi/exps"], arrays[f"{name}/A_lo/exps"]])
    ref_eb = np.concatenate([arrays[f"{name}/B_hi/exps"], arrays[f"{name}/B_lo/exps"]])
    finite = np.isfinite(np.concatenate([ref_ea, ref_eb], axis=1).astype(np.float64))
    assert np.array_equal(ea, ref_ea.astype(np.int32))
    assert np.array_equal(eb, ref_eb.astype(np.int32))
    assert finite.all()


@pytest.mark.parametrize("shape,seed,wide", [((300, 2000), 1, False), ((256, 8192), 2, False),
                                             ((97, 4100), 3, True), ((2, 70000), 4, False),
                                             ((300, 12000), 8, True), ((41, 3001), 9, False),
                                             ((700, 1026), 10, True), ((33, 16000), 11, True),
                                             ((50, 20000), 12, False), ((40, 40000), 13, True)])
def test_rows_match_oracle(shape, seed, wide):
    rng = np.random.RandomState(seed)
    X = rng.randn(*shape)
    if wide:
        X = (rng.rand(*shape) - 0.5) * np.exp(10 * rng.randn(*shape))
    rho = O.compute_rho_f32(shape[1])
    for n_hi, n_lo in ((4, 1), (5, 4), (3, 1)):
        s, e, st = dev_extract(X, rho, n_hi, n_lo, axis=1)
        hi, lo = O.double_f32_split(X)
        rs, re_ = O.extract_rows_f32(hi, rho, n_hi)
        ls, le = O.extract_rows_f32(lo, rho, n_lo)
        assert st == 0
        assert same_bits(bf16_bits_to_f32(s), np.stack(rs + ls))
        assert np.array_equal(e, np.stack(re_ + le).astype(np.int32))


@pytest.mark.parametrize("shape,seed", [((2000, 300), 5), ((8192, 96), 6), ((4100, 33), 7)])
def test_cols_match_oracle(shape, seed):
    rng = np.random.RandomState(seed)
    X = rng.randn(*shape)
    rho = O.compute_rho_f32(shape[0])
    s, e, st = dev_extract(X, rho, 4, 1, axis=0)
    hi, lo = O.double_f32_split(X)
    cs, ce = O.extract_cols_f32(hi, rho, 4)
    ls, le = O.extract_cols_f32(lo, rho, 1)
    assert st == 0
    assert same_bits(bf16_bits_to_f32(s), np.stack(cs + ls).transpose(0, 2, 1))
    assert np.array_equal(e, np.stack(ce + le).astype(np.int32))


def test_nonfinite_and_range_flags():
    from ozaki_jax_b200 import _lib
    X = np.ones((4, 100))
    X[2, 7] = np.nan
    _, _, st = dev_extract(X, 17, 4, 1, axis=1)
    assert st & _lib.OZK_FLAG_NONFINITE
    X = np.ones((100, 4))
    X[3, 1] = np.inf
    _, _, st = dev_extract(X, 17, 4, 1, axis=0)
    assert st & _lib.OZK_FLAG_NONFINITE
    X = np.ones((4, 100))
    X[1, 1] = 1e300
    _, _, st = dev_extract(X, 17, 4, 1, axis=1)
    assert st == _lib.OZK_FLAG_RANGE
