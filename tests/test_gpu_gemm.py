"""K2 parity through the C ABI: exact per-pair products, the reference's 2Sum
words bit for bit, and the FP64 epilogue within tolerance of the oracle."""

import ctypes

import numpy as np
import pytest
import torch

import ozaki_oracle as O
from conftest import same_bits

pytestmark = pytest.mark.gpu

PRESETS = {"high": (4, 1), "medium": (3, 1), "max": (5, 4), "c42": (4, 2)}


def lib():
    from ozaki_jax_b200 import _lib
    return _lib


def pairs_arrays(n_hi, n_lo):
    pa = (ctypes.c_uint8 * 256)()
    pb = (ctypes.c_uint8 * 256)()
    n = lib().load().ozk_pair_schedule(n_hi, n_lo, pa, pb, 256)
    return pa, pb, n


def device_slices(A, B, n_hi, n_lo):
    from ozaki_jax_b200.extract import extract_device
    Ad = torch.as_tensor(A).cuda()
    Bd = torch.as_tensor(B).cuda()
    rho = O.compute_rho_f32(A.shape[1])
    SA, k_pad, eA, _ = extract_device(Ad, rho, n_hi, n_lo, 1)
    SB, _, eB, _ = extract_device(Bd, rho, n_hi, n_lo, 0)
    return SA, SB, eA, eB, k_pad


def run_products(SA, SB, eA, eB, k_pad, n_hi, n_lo):
    L = lib()
    nS = n_hi + n_lo
    N, M = SA.shape[1], SB.shape[1]
    pa, pb, n = pairs_arrays(n_hi, n_lo)
    P = torch.full((n, N, M), float("nan"), dtype=torch.float32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.load().ozk_slice_gemm(SA.data_ptr(), eA.data_ptr(), nS, SB.data_ptr(), eB.data_ptr(),
                                 nS, N, M, k_pad, pa, pb, n, L.OZK_ACC_PRODUCTS, 0, 1.0, 0.0,
                                 None, 0, None, 0, P.data_ptr(), None, 0, 0, st.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    L.check(rc)
    torch.cuda.synchronize()
    assert st.item() == 0
    return P.cpu().numpy()


@pytest.mark.parametrize("N,K,M", [(128, 64, 128), (256, 1024, 192), (200, 3000, 72),
                                   (129, 257, 65), (1, 128, 1), (128, 8192, 16)])
def test_products_bit_exact(N, K, M):
    rng = np.random.RandomState(N + K + M)
    A, B = rng.randn(N, K), rng.randn(K, M)
    SA, SB, eA, eB, k_pad = device_slices(A, B, 4, 1)
    P = run_products(SA, SB, eA, eB, k_pad, 4, 1)
    sa, _, sb, _, _ = O.extract_ondevice(A, B, 4, 1)
    pairs, _, _ = O.ondevice_pairs(4, 1)
    ref = O.slice_products(sa, sb, pairs)
    assert same_bits(P, ref)


def test_products_exact_at_the_bound():
    """Every slice at the largest magnitude the K bound allows (K = 8192, 5-bit
    slices): partial sums reach 2^23 grid units and must stay exact."""
    K, N, M = 8192, 128, 128
    rng = np.random.RandomState(11)
    v = np.float32(31.0 / 16.0)
    sa = (rng.choice([-1, 1], size=(1, N, K)) * v).astype(np.float32)
    sb = (rng.choice([-1, 1], size=(1, M, K)) * v).astype(np.float32)
    sa[0, 0, :] = v
    sb[0, 0, :] = v  # one output at exactly K * (31/16)^2
    to_bits = lambda x: torch.as_tensor((x.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)).cuda()
    SA, SB = to_bits(sa), to_bits(sb)
    e = torch.zeros((1, N), dtype=torch.int32, device="cuda")
    L = lib()
    pa = (ctypes.c_uint8 * 1)(0)
    pb = (ctypes.c_uint8 * 1)(0)
    P = torch.empty((1, N, M), dtype=torch.float32, device="cuda")
    L.check(L.load().ozk_slice_gemm(SA.data_ptr(), e.data_ptr(), 1, SB.data_ptr(), e.data_ptr(), 1,
                                    N, M, K, pa, pb, 1, L.OZK_ACC_PRODUCTS, 0, 1.0, 0.0, None, 0,
                                    None, 0, P.data_ptr(), None, 0, 0, None,
                                    torch.cuda.current_stream().cuda_stream))
    exact = sa[0].astype(np.float64) @ sb[0].astype(np.float64).T
    got = P.cpu().numpy()[0].astype(np.float64)
    assert np.array_equal(got, exact)
    assert got[0, 0] == K * (31.0 / 16.0) ** 2


@pytest.mark.parametrize("name", ["n64_s0", "rect_37x100x23", "zeros_24x48x16",
                                  "wide_phi10_40x96x32", "k1040_8x1040x8", "log2_edges_12x20x10",
                                  "vec_1x128x1", "outer_48x1x40", "scales_16x32x12"])
def test_ondevice_accumulation_bit_exact_with_reference(golden, name):
    """accumulation='ondevice' (products + reference-order 2Sum) reproduces the
    reference's fused result bit for bit, for every preset."""
    from ozaki_jax_b200.matmul import _ondevice_device
    arrays, _ = golden
    A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
    for pname, (n_hi, n_lo) in PRESETS.items():
        key = f"{name}/{pname}/fused"
        if key not in arrays:
            continue
        C, st = _ondevice_device(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), n_hi, n_lo,
                                 "ondevice")
        assert same_bits(C.cpu().numpy(), arrays[key]), pname


def test_accumulate_2sum_words_bit_exact(golden):
    arrays, _ = golden
    L = lib()
    for name in ("n64_s0", "rect_37x100x23", "wide_phi10_40x96x32"):
        A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
        for pname in ("high", "max"):
            n_hi, n_lo = PRESETS[pname]
            SA, SB, eA, eB, k_pad = device_slices(A, B, n_hi, n_lo)
            P = run_products(SA, SB, eA, eB, k_pad, n_hi, n_lo)
            N, M = A.shape[0], B.shape[1]
            Pd = torch.as_tensor(P).cuda()
            ch = torch.empty((N, M), dtype=torch.float32, device="cuda")
            cl = torch.empty_like(ch)
            L.check(L.load().ozk_accumulate_2sum(Pd.data_ptr(), eA.data_ptr(), eB.data_ptr(), N, M,
                                                 n_hi, n_lo, ch.data_ptr(), cl.data_ptr(), None, 0,
                                                 torch.cuda.current_stream().cuda_stream))
            assert same_bits(ch.cpu().numpy(), arrays[f"{name}/{pname}/C_hi"])
            assert same_bits(cl.cpu().numpy(), arrays[f"{name}/{pname}/C_lo"])


FP64_CASES = ["n64_s0", "rect_37x100x23", "zeros_24x48x16", "wide_phi10_40x96x32",
              "k1040_8x1040x8", "vec_1x128x1", "outer_48x1x40"]


@pytest.mark.parametrize("name", FP64_CASES)
def test_fp64_epilogue_matches_fp64_oracle(golden, name):
    """accumulation='host' (FP64 sums) agrees with the reference's
    FP64-accumulating NumPy pipeline (matmul_numpy, goldens) to FP64 rounding
    element by element: the two differ only in the order of exact-product
    additions."""
    from ozaki_jax_b200.matmul import _ondevice_device
    arrays, _ = golden
    A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
    E = O.exact_product(A, B)
    for pname, (n_hi, n_lo) in PRESETS.items():
        key = f"{name}/{pname}/numpy"
        if key not in arrays:
            continue
        C, _ = _ondevice_device(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), n_hi, n_lo,
                                "host")
        C = C.cpu().numpy()
        ref = arrays[key]
        scale = np.abs(A) @ np.abs(B)
        assert np.all(np.abs(C - ref) <= 64 * 2.0 ** -52 * scale + 1e-300), pname
        # accuracy no worse than 1.5x the reference's; below 32 ulps of FP64 the
        # Ozaki truncation is gone and only FP64 summation order remains
        e_ref = min(O.rel_err(ref, E), O.rel_err(arrays[f"{name}/{pname}/fused"], E))
        assert O.rel_err(C, E) <= max(1.5 * e_ref, 32 * 2.0 ** -52), pname


@pytest.mark.parametrize("name", FP64_CASES)
def test_fixed_point_epilogue_error_model(golden, name):
    """accumulation='fused' (exact int64 fixed-point sums): normwise accuracy
    no worse than 1.5x the reference's, and element by element within the
    fixed-point resolution of the reference's FP64 pipeline -- a few units of
    2^-50 * max|A[r,:]| * max|B[:,c]| per term (the same row/column-max scale
    the Ozaki truncation error has)."""
    from ozaki_jax_b200.matmul import _ondevice_device
    arrays, _ = golden
    A, B = arrays[f"{name}/A"], arrays[f"{name}/B"]
    E = O.exact_product(A, B)
    rmax = np.max(np.abs(A), axis=1)[:, None]
    cmax = np.max(np.abs(B), axis=0)[None, :]
    for pname, (n_hi, n_lo) in PRESETS.items():
        key = f"{name}/{pname}/numpy"
        if key not in arrays:
            continue
        C, _ = _ondevice_device(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), n_hi, n_lo,
                                "fused")
        C = C.cpu().numpy()
        ref = arrays[key]
        n_pairs = n_hi * n_hi + 2 * n_hi * n_lo
        bound = n_pairs * 2.0 ** -48 * rmax * cmax + 64 * 2.0 ** -52 * (np.abs(A) @ np.abs(B))
        assert np.all(np.abs(C - ref) <= bound + 1e-300), pname
        e_ref = min(O.rel_err(ref, E), O.rel_err(arrays[f"{name}/{pname}/fused"], E))
        assert O.rel_err(C, E) <= max(1.5 * e_ref, 32 * 2.0 ** -52), pname


def test_accuracy_gate_256x8192x256(golden):
    """North-star gate at K = 8192: error vs the FP64 product no worse than
    1.5x the reference's own error at the same preset (golden_meta)."""
    from ozaki_jax_b200.matmul import _ondevice_device
    _, meta = golden
    rng = np.random.RandomState(0)
    A = rng.randn(256, 8192)
    B = rng.randn(8192, 256)
    R = A @ B
    for pname in ("high", "medium", "max"):
        n_hi, n_lo = PRESETS[pname]
        C, _ = _ondevice_device(torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda(), n_hi, n_lo,
                                "fused")
        err = float(np.linalg.norm(C.cpu().numpy() - R) / np.linalg.norm(R))
        ref = meta["ref_err_256x8192x256"][pname]["numpy"]
        assert err <= 1.5 * ref, (pname, err, ref)


def test_wide_range_max_preset_config_c3():
    """The wide-range 'max' workload in miniature: (U(0,1)-0.5)*exp(10 N(0,1))
    entries, K = 8192 (int8 codes, 256-wide tiles).  Per-row scaling truncates the
    small entries of a row, so the reference's own error is large (about 1e-6);
    'fused' must stay within 1.5x of the reference's matmul_numpy error against
    the exact product, and 'ondevice' must be the reference's fused result bit
    for bit."""
    from ozaki_jax_b200.matmul import _ondevice_device
    rng = np.random.RandomState(0)
    n, k, m = 256, 8192, 256
    A = (rng.rand(n, k) - 0.5) * np.exp(10 * rng.randn(n, k))
    B = (rng.rand(k, m) - 0.5) * np.exp(10 * rng.randn(k, m))
    E = O.exact_product(A, B)
    ref_err = O.rel_err(O.ondevice_numpy(A, B, 5, 4), E)
    Ad, Bd = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
    C, st = _ondevice_device(Ad, Bd, 5, 4, "fused")
    torch.cuda.synchronize()
    assert st.item() == 0
    err = O.rel_err(C.cpu().numpy(), E)
    assert err <= 1.5 * ref_err, (err, ref_err)
    C2, _ = _ondevice_device(Ad, Bd, 5, 4, "ondevice")
    _, _, ref_fused = O.fused_ondevice(A, B, 5, 4)
    assert same_bits(C2.cpu().numpy(), ref_fused)
