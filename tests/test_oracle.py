"""The oracle is pinned to golden vectors made by the reference's own code.

Bit-exact: slices, exponents, the 2Sum (C_hi, C_lo) words and the FP64
results of the reference's NumPy pipelines.
"""

import numpy as np
import pytest

import ozaki_oracle as O
from conftest import bf16_bits_to_f32, same_bits

CASES = ["n64_s0", "rect_37x100x23", "zeros_24x48x16", "wide_phi10_40x96x32",
         "k1040_8x1040x8", "scales_16x32x12", "log2_edges_12x20x10", "vec_1x128x1",
         "outer_48x1x40"]
PRESETS = {"high": (4, 1), "medium": (3, 1), "max": (5, 4), "c42": (4, 2)}


def test_rho_tables(golden):
    _, meta = golden
    for K, rho in meta["rho_f32"].items():
        assert O.compute_rho_f32(int(K)) == rho, K
    for K, rho in meta["rho_f64"].items():
        assert O.compute_rho_f64(int(K)) == rho, K


def test_pair_schedules(golden):
    _, meta = golden
    for key, ref in meta["pair_schedule"].items():
        n_hi, n_lo = map(int, key.split(","))
        pairs, groups, bounds = O.ondevice_pairs(n_hi, n_lo)
        assert [a for a, _ in pairs] == ref["pair_a"]
        assert [b for _, b in pairs] == ref["pair_b"]
        assert len(pairs) == ref["n_pairs"] == n_hi * n_hi + 2 * n_hi * n_lo
        assert [[a, ps] for a, ps in groups] == ref["groups"]
        assert list(bounds) == ref["bounds"]


@pytest.mark.parametrize("name", CASES)
def test_extraction_bit_exact(golden, name):
    arrays, meta = golden
    A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
    rho = meta["cases"][name]["rho"]
    assert O.compute_rho_f32(A.shape[1]) == rho
    A_hi, A_lo = O.double_f32_split(A)
    B_hi, B_lo = O.double_f32_split(B)
    for part, X, fn in (("A_hi", A_hi, O.extract_rows_f32), ("A_lo", A_lo, O.extract_rows_f32),
                        ("B_hi", B_hi, O.extract_cols_f32), ("B_lo", B_lo, O.extract_cols_f32)):
        s, e = fn(X, rho, 5)
        ref_s = bf16_bits_to_f32(arrays[f"{name}/{part}/slices"])
        assert same_bits(np.stack(s), ref_s), part
        assert np.array_equal(np.stack(e), arrays[f"{name}/{part}/exps"].astype(np.float32)), part


@pytest.mark.parametrize("name", CASES)
def test_pipelines_bit_exact(golden, name):
    arrays, meta = golden
    A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
    for pname, prec in PRESETS.items():
        if f"{name}/{pname}/fused" not in arrays:
            continue
        ch, cl, c = O.fused_ondevice(A, B, *prec)
        assert same_bits(ch, arrays[f"{name}/{pname}/C_hi"]), pname
        assert same_bits(cl, arrays[f"{name}/{pname}/C_lo"]), pname
        assert same_bits(c, arrays[f"{name}/{pname}/fused"]), pname
        with np.errstate(all="ignore"):
            cn = O.ondevice_numpy(A, B, *prec)
        assert same_bits(cn, arrays[f"{name}/{pname}/numpy"]), pname
    if f"{name}/host8" in arrays:
        assert same_bits(O.host_numpy(A, B, 8), arrays[f"{name}/host8"])
    else:
        rep = O.host_safety_report(A, B, 8)
        assert not rep["safe"]
        assert meta["cases"][name]["host8_error"].endswith("; ".join(rep["reasons"]))


def test_gram_residual_bit_exact(golden):
    arrays, _ = golden
    G_A = arrays["gram/A"]
    for pname in ("high", "medium"):
        G = O.gram_ozaki(G_A, *PRESETS[pname])
        for acc in ("bf16_interleaved", "fused"):
            assert same_bits(G, arrays[f"gram/{pname}/{acc}"]), (pname, acc)
    A, x, b = arrays["residual/A"], arrays["residual/x"], arrays["residual/b"]
    for pname in ("high", "medium"):
        r = O.residual_ozaki(A, x, b, *PRESETS[pname])
        for acc in ("bf16_interleaved", "fused"):
            assert same_bits(r, arrays[f"residual/{pname}/{acc}"]), (pname, acc)
    rv = O.residual_ozaki(A, arrays["residual/xv"], arrays["residual/bv"])
    assert same_bits(rv, arrays["residual/high/vec"])


def test_preflight_messages(golden):
    _, meta = golden
    msgs = meta["messages"]
    prefix = "Ozaki preflight marked this input as unsafe: "
    rep = O.ondevice_safety_report(np.full((4, 4), np.nan), np.ones((4, 4)), 4, 1)
    assert msgs["ondevice_nan"] == prefix + "; ".join(rep["reasons"])
    rng = np.random.RandomState(9)
    A, B = rng.randn(2, 10000), rng.randn(10000, 2)
    rep = O.host_safety_report(A, B, 8)
    assert msgs["host_k10000"] == prefix + "; ".join(rep["reasons"])


def test_exact_product_reference():
    rng = np.random.RandomState(0)
    A, B = rng.randn(64, 64), rng.randn(64, 64)
    E = O.exact_product(A, B)
    # BLAS FP64 is within a few ulps of the correctly rounded product
    assert O.rel_err(A @ B, E) < 1e-15
    assert O.rel_err(O.host_numpy(A, B), E) < 1e-14


def test_int8_code_is_the_low_byte_of_the_sum():
    """The identity the device extraction uses for its int8 codes, checked in
    NumPy float32 (IEEE round to nearest even): for rho >= 19 and every slice
    exponent c in [-127, 127 - rho], sigma = 0.75 * 2^(rho+c) has a zero low
    byte, and for a residual |r| < 2^(c+1) the code bits(RN(r + sigma)) -
    bits(sigma) lies in [-2^(25-rho), 2^(25-rho)], equals the low byte of
    bits(RN(r + sigma)) read as int8, and times 2^(rho+c-24) is the slice value
    RN(RN(r + sigma) - sigma) of the reference's recurrence
    (ozaki_jax/extract.py:116-154)."""
    rng = np.random.RandomState(5)
    for rho in range(19, 25):
        for c in range(-127, 128 - rho):
            sig = np.float32(0.75 * 2.0 ** (rho + c))
            sb = int(sig.view(np.uint32))
            assert sb & 0xFF == 0
            r = (rng.uniform(-1.0, 1.0, 64) * 2.0 ** (c + 1)).astype(np.float32)
            r = r[np.abs(r.astype(np.float64)) < 2.0 ** (c + 1)]
            r = np.concatenate([r, np.float32([0.0, -0.0])])
            t = (r + sig).astype(np.float32)
            tb = t.view(np.uint32).astype(np.int64)
            code = tb - sb
            assert np.all(np.abs(code) <= 2 ** (25 - rho)), (rho, c)
            low = (tb & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
            assert np.array_equal(low, code), (rho, c)
            v = (t - sig).astype(np.float32)
            assert np.array_equal(v.astype(np.float64), code * 2.0 ** (rho + c - 24)), (rho, c)
