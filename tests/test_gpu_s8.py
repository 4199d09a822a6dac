"""int8 slice codes and the kind::i8 slice GEMM against the BF16 path.

For rho >= 19 every BF16 slice is an exact int8 code times 2^(rho-24), and
the int8 x int8 -> int32 products equal the BF16 -> FP32 products exactly, so
every fixed-point result must match the BF16 path bit for bit: the standalone
entry points, matmul / gram through the pipelines (which pick int8 on their
own), and the gated BF16 recomputation when some slice has no int8 code."""

import ctypes

import numpy as np
import pytest
import torch

import ozaki_oracle as O
from ozaki_jax_b200 import _lib as L
from ozaki_jax_b200.extract import extract_device

pytestmark = pytest.mark.gpu


def stream():
    return torch.cuda.current_stream().cuda_stream


def snake(n_hi, n_lo):
    pa = (ctypes.c_uint8 * 256)()
    pb = (ctypes.c_uint8 * 256)()
    n = L.load().ozk_pair_schedule_snake(n_hi, n_lo, pa, pb, 256)
    return pa, pb, n


def s8_slices(X, rho, n_hi, n_lo, axis):
    """int8 codes through the C ABI: (codes [ns][lines][k8], k8, exps, fail)."""
    lib = L.load()
    Xd = torch.as_tensor(X).cuda()
    lines, K = (X.shape if axis == 1 else X.shape[::-1])
    k8 = (K + 127) // 128 * 128
    ns = n_hi + n_lo
    codes = torch.full((ns, lines, k8), 99, dtype=torch.int8, device="cuda")
    exps = torch.empty((ns, lines), dtype=torch.int32, device="cuda")
    fail = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    if axis == 1:
        L.check(lib.ozk_extract_rows_s8_f64(Xd.data_ptr(), K, lines, K, rho, n_hi, n_lo,
                                            codes.data_ptr(), k8, exps.data_ptr(), fail.data_ptr(),
                                            st.data_ptr(), stream()))
    else:
        L.check(lib.ozk_extract_cols_s8_f64(Xd.data_ptr(), lines, K, lines, rho, n_hi, n_lo,
                                            codes.data_ptr(), k8, exps.data_ptr(), None, 0,
                                            fail.data_ptr(), st.data_ptr(), stream()))
    torch.cuda.synchronize()
    return codes, k8, exps, int(fail.item())


def bf16_values(bits):
    b = bits.cpu().numpy().astype(np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


@pytest.mark.parametrize("axis", [1, 0])
@pytest.mark.parametrize("K,n_hi,n_lo", [(4097, 4, 1), (8192, 3, 1), (5000, 5, 4), (12000, 4, 1),
                                         (20000, 4, 1), (32768, 4, 1), (40000, 3, 2)])
def test_codes_are_the_bf16_slices(axis, K, n_hi, n_lo):
    rng = np.random.RandomState(K + axis)
    lines = 300
    X = rng.randn(lines, K) if axis == 1 else rng.randn(K, lines)
    X *= np.exp(rng.randn(*X.shape) * 2)
    rho = O.compute_rho_f32(K)
    assert rho >= 19
    codes, k8, e8, fail = s8_slices(X, rho, n_hi, n_lo, axis)
    assert fail == 0
    S16, k_pad, e16, _ = extract_device(torch.as_tensor(X).cuda(), rho, n_hi, n_lo, axis)
    torch.cuda.synchronize()
    assert torch.equal(e8, e16)
    vals = bf16_values(S16)[:, :, :K]
    q = codes.cpu().numpy().astype(np.float64)
    assert np.abs(q).max() <= 64
    assert np.array_equal(q[:, :, :K], vals.astype(np.float64) * 2.0 ** (24 - rho))
    assert np.all(q[:, :, K:] == 0)


@pytest.mark.parametrize("K", [700, 1024, 1025, 2048, 2049, 3000, 4096, 5000, 8192, 8193, 16384])
@pytest.mark.parametrize("ldx", [20, 21])
def test_column_codes_against_oracle_strided(K, ldx):
    """int8 column codes of a strided K x 13 operand (even and odd leading
    dimensions, a zero column) against the oracle's column extraction, from
    short columns (rho 19 forced where the policy gives less) to 16384 rows."""
    rng = np.random.RandomState(K + ldx)
    cols, n_hi, n_lo = 13, 4, 1
    Xbig = rng.randn(K, ldx) * np.exp(rng.randn(K, ldx) * 2)
    Xbig[:, 6] = 0.0  # a zero column
    X = Xbig[:, :cols]
    rho = max(19, O.compute_rho_f32(K))
    lib = L.load()
    Xd = torch.as_tensor(Xbig).cuda()
    k8 = (K + 127) // 128 * 128
    codes = torch.full((5, cols, k8), 99, dtype=torch.int8, device="cuda")
    exps = torch.empty((5, cols), dtype=torch.int32, device="cuda")
    fail = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(lib.ozk_extract_cols_s8_f64(Xd.data_ptr(), ldx, K, cols, rho, n_hi, n_lo,
                                        codes.data_ptr(), k8, exps.data_ptr(), None, 0,
                                        fail.data_ptr(), st.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert fail.item() == 0 and st.item() == 0
    hi, lo = O.double_f32_split(X)
    sh, eh = O.extract_cols_f32(hi, rho, n_hi)
    sl, el = O.extract_cols_f32(lo, rho, n_lo)
    ref = np.stack([np.asarray(v, dtype=np.float64).T for v in list(sh) + list(sl)])
    q = codes.cpu().numpy().astype(np.float64)
    assert np.array_equal(q[:, :, :K], ref * 2.0 ** (24 - rho))
    assert np.all(q[:, :, K:] == 0)
    assert np.array_equal(exps.cpu().numpy(), np.stack(list(eh) + list(el)).astype(np.int32))


@pytest.mark.parametrize("K,lines,n_hi,n_lo", [(16400, 400, 4, 1), (20000, 300, 3, 1),
                                               (32768, 300, 4, 1), (65536, 150, 4, 1),
                                               (24000, 160, 5, 4)])
def test_long_row_codes_against_oracle(K, lines, n_hi, n_lo):
    """int8 row codes of rows that a cluster of CTAs holds together (clusters
    of 4096- or 8192-column CTAs exchanging line maxima), with more rows than
    resident clusters, so each cluster goes through several rows and the
    exchange's tags and parity slots are reused: codes and exponents against
    the oracle's row extraction on every row.  Rows of very different scales,
    a zero row; 16400 columns leave three CTAs of each cluster without
    columns."""
    rng = np.random.RandomState(K + lines)
    X = rng.randn(lines, K) * np.exp(rng.randn(lines, 1) * 8)
    X *= np.exp(rng.randn(lines, K))
    X[lines // 3] = 0.0  # a zero row
    rho = O.compute_rho_f32(K)
    codes, k8, exps, fail = s8_slices(X, rho, n_hi, n_lo, 1)
    assert fail == 0
    hi, lo = O.double_f32_split(X)
    sh, eh = O.extract_rows_f32(hi, rho, n_hi)
    sl, el = O.extract_rows_f32(lo, rho, n_lo)
    q = codes.cpu().numpy()
    for t, ref in enumerate(list(sh) + list(sl)):
        assert np.array_equal(q[t, :, :K].astype(np.float64),
                              np.asarray(ref, dtype=np.float64) * 2.0 ** (24 - rho)), t
    assert np.all(q[:, :, K:] == 0)
    assert np.array_equal(exps.cpu().numpy(), np.stack(list(eh) + list(el)).astype(np.int32))


@pytest.mark.parametrize("K,lines,n_hi,n_lo", [(6001, 301, 4, 1), (8192, 3, 3, 1),
                                               (4500, 1, 4, 2), (7000, 600, 4, 1)])
def test_column_codes_odd_counts(K, lines, n_hi, n_lo):
    """Column codes for odd, single and many columns, with a zero column:
    codes and exponents must be the BF16 column slices'."""
    rng = np.random.RandomState(K + lines)
    X = rng.randn(K, lines) * np.exp(rng.randn(K, lines) * 2)
    X[:, lines // 2] = 0.0  # a zero column
    rho = O.compute_rho_f32(K)
    codes, k8, e8, fail = s8_slices(X, rho, n_hi, n_lo, 0)
    assert fail == 0
    S16, _, e16, _ = extract_device(torch.as_tensor(X).cuda(), rho, n_hi, n_lo, 0)
    torch.cuda.synchronize()
    assert torch.equal(e8, e16)
    vals = bf16_values(S16)[:, :, :K]
    q = codes.cpu().numpy().astype(np.float64)
    assert np.array_equal(q[:, :, :K], vals.astype(np.float64) * 2.0 ** (24 - rho))
    assert np.all(q[:, :, K:] == 0)


@pytest.mark.parametrize("axis", [1, 0])
@pytest.mark.parametrize("bad,flag", [(np.nan, L.OZK_FLAG_NONFINITE),
                                      (np.inf, L.OZK_FLAG_NONFINITE),
                                      (1e300, L.OZK_FLAG_RANGE)])
def test_int8_extraction_flags_one_bad_value(axis, bad, flag):
    """One non-finite or out-of-range value among finite ones (its neighbour
    in the same packed pair is finite) raises its flag in the status word."""
    rng = np.random.RandomState(3)
    X = rng.randn(64, 6000) if axis == 1 else rng.randn(6000, 64)
    X[(5, 1001) if axis == 1 else (1001, 5)] = bad
    lib = L.load()
    Xd = torch.as_tensor(X).cuda()
    lines, K = (X.shape if axis == 1 else X.shape[::-1])
    k8 = (K + 127) // 128 * 128
    codes = torch.empty((5, lines, k8), dtype=torch.int8, device="cuda")
    exps = torch.empty((5, lines), dtype=torch.int32, device="cuda")
    fail = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rho = O.compute_rho_f32(K)
    if axis == 1:
        L.check(lib.ozk_extract_rows_s8_f64(Xd.data_ptr(), K, lines, K, rho, 4, 1,
                                            codes.data_ptr(), k8, exps.data_ptr(), fail.data_ptr(),
                                            st.data_ptr(), stream()))
    else:
        L.check(lib.ozk_extract_cols_s8_f64(Xd.data_ptr(), lines, K, lines, rho, 4, 1,
                                            codes.data_ptr(), k8, exps.data_ptr(), None, 0,
                                            fail.data_ptr(), st.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert int(st.item()) & flag


def bf16_fixed_gemm(SA, eA, SB, eB, k_pad, N, M, rho, n_hi, n_lo, symmetric=0, alpha=1.0,
                    beta=0.0, Cin=None):
    lib = L.load()
    pa, pb, n = snake(n_hi, n_lo)
    C = torch.full((N, M), float("nan"), dtype=torch.float64, device="cuda")
    GW = torch.empty(lib.ozk_slice_gemm_workspace_bytes(), dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(lib.ozk_slice_gemm(SA.data_ptr(), eA.data_ptr(), n_hi + n_lo, SB.data_ptr(),
                               eB.data_ptr(), n_hi + n_lo, N, M, k_pad, pa, pb, n, L.OZK_ACC_FIXED,
                               symmetric, alpha, beta, None if Cin is None else Cin.data_ptr(), M,
                               C.data_ptr(), M, None, GW.data_ptr(), GW.numel(), rho,
                               st.data_ptr(), stream()))
    torch.cuda.synchronize()
    return C.cpu().numpy()


def s8_fixed_gemm(SA, eA, SB, eB, k8, N, M, rho, n_hi, n_lo, symmetric=0, alpha=1.0, beta=0.0,
                  Cin=None, skip=None):
    lib = L.load()
    pa, pb, n = snake(n_hi, n_lo)
    C = torch.full((N, M), -3.0, dtype=torch.float64, device="cuda")
    GW = torch.empty(lib.ozk_slice_gemm_workspace_bytes(), dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(lib.ozk_slice_gemm_s8(SA.data_ptr(), eA.data_ptr(), n_hi + n_lo, SB.data_ptr(),
                                  eB.data_ptr(), n_hi + n_lo, N, M, k8, pa, pb, n, symmetric,
                                  alpha, beta, None if Cin is None else Cin.data_ptr(), M,
                                  C.data_ptr(), M, GW.data_ptr(), GW.numel(), rho,
                                  None if skip is None else skip.data_ptr(), st.data_ptr(),
                                  stream()))
    torch.cuda.synchronize()
    assert st.item() == 0
    return C.cpu().numpy()


def same(a, b):
    return np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(
        np.nan_to_num(a, nan=0.0).view(np.int64), np.nan_to_num(b, nan=0.0).view(np.int64))


# The last three shapes leave a sparse last wave of 256 x 256 tiles on the 74
# CTA pairs of a B200 (26 of 100, 36 and 16 tiles), so those tiles' pair lists
# are cut into 2, 2 and 4 chunks on different units and the int64 partial sums
# combined: still bit for bit the BF16 result.
@pytest.mark.parametrize("N,K,M,n_hi,n_lo", [(256, 4224, 256, 4, 1), (520, 6000, 300, 4, 1),
                                             (384, 8192, 640, 3, 1), (300, 5000, 260, 5, 4),
                                             (2560, 4224, 2560, 4, 1), (1536, 4224, 1536, 5, 4),
                                             (1024, 8192, 1024, 3, 1)])
def test_s8_gemm_matches_bf16_gemm(N, K, M, n_hi, n_lo):
    rng = np.random.RandomState(N * 7 + M)
    A = rng.randn(N, K) * np.exp(rng.randn(N, 1) * 3)
    B = rng.randn(K, M) * np.exp(rng.randn(1, M) * 3)
    rho = O.compute_rho_f32(K)
    SA8, k8, eA, fa = s8_slices(A, rho, n_hi, n_lo, 1)
    SB8, _, eB, fb = s8_slices(B, rho, n_hi, n_lo, 0)
    assert fa == 0 and fb == 0
    C8 = s8_fixed_gemm(SA8, eA, SB8, eB, k8, N, M, rho, n_hi, n_lo)
    SA, k_pad, eA2, _ = extract_device(torch.as_tensor(A).cuda(), rho, n_hi, n_lo, 1)
    SB, _, eB2, _ = extract_device(torch.as_tensor(B).cuda(), rho, n_hi, n_lo, 0)
    C16 = bf16_fixed_gemm(SA, eA2, SB, eB2, k_pad, N, M, rho, n_hi, n_lo)
    assert same(C8, C16)
    # residual form (alpha = -1, beta = 1) and the skip word
    Bv = torch.as_tensor(rng.randn(N, M)).cuda()
    R8 = s8_fixed_gemm(SA8, eA, SB8, eB, k8, N, M, rho, n_hi, n_lo, alpha=-1.0, beta=1.0, Cin=Bv)
    R16 = bf16_fixed_gemm(SA, eA2, SB, eB2, k_pad, N, M, rho, n_hi, n_lo, alpha=-1.0, beta=1.0,
                          Cin=Bv)
    assert same(R8, R16)
    skip = torch.ones(1, dtype=torch.int32, device="cuda")
    assert np.all(s8_fixed_gemm(SA8, eA, SB8, eB, k8, N, M, rho, n_hi, n_lo, skip=skip) == -3.0)


@pytest.mark.parametrize("K", [384, 3328])  # 3328: 91 upper-triangle tiles, 17 split in 4
def test_s8_symmetric_gram_tiles(K):
    rng = np.random.RandomState(2)
    N = 5000  # G = A^T A: lines are the K columns of A, length N
    A = rng.randn(N, K)
    rho = O.compute_rho_f32(N)
    S8, k8, e8, fail = s8_slices(A, rho, 4, 1, 0)
    assert fail == 0
    G8 = s8_fixed_gemm(S8, e8, S8, e8, k8, K, K, rho, 4, 1, symmetric=1)
    S16, k_pad, e16, _ = extract_device(torch.as_tensor(A).cuda(), rho, 4, 1, 0)
    G16 = bf16_fixed_gemm(S16, e16, S16, e16, k_pad, K, K, rho, 4, 1, symmetric=1)
    assert same(G8, G16)
    assert np.array_equal(G8, G8.T)


def bf16_pipeline(A, B, n_hi, n_lo):
    """matmul with fixed-point sums on BF16 slices only (standalone entry points)."""
    rho = O.compute_rho_f32(A.shape[1])
    SA, k_pad, eA, _ = extract_device(torch.as_tensor(A).cuda(), rho, n_hi, n_lo, 1)
    SB, _, eB, _ = extract_device(torch.as_tensor(B).cuda(), rho, n_hi, n_lo, 0)
    return bf16_fixed_gemm(SA, eA, SB, eB, k_pad, A.shape[0], B.shape[1], rho, n_hi, n_lo)


def pipeline(A, B, n_hi=4, n_lo=1):
    lib = L.load()
    Ad, Bd = torch.as_tensor(A).cuda(), torch.as_tensor(B).cuda()
    N, K = A.shape
    M = B.shape[1]
    C = torch.empty((N, M), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(lib.ozk_matmul_f64(Ad.data_ptr(), K, Bd.data_ptr(), M, C.data_ptr(), M, N, K, M, -1,
                               n_hi, n_lo, L.OZK_ACC_FIXED, None, 0, st.data_ptr(), stream()))
    torch.cuda.synchronize()
    return C.cpu().numpy(), int(st.item())


def test_pipeline_takes_s8_and_matches_bf16():
    rng = np.random.RandomState(8)
    A, B = rng.randn(600, 4500), rng.randn(4500, 520)
    C, st = pipeline(A, B)
    assert st == 0
    assert same(C, bf16_pipeline(A, B, 4, 1))


@pytest.mark.parametrize("side", ["A row", "B column"])
@pytest.mark.parametrize("scale", [2.0 ** -135, 2.0 ** 112])
def test_unrepresentable_slices_fall_back_on_device(scale, side):
    """A row of A (or a column of B) whose slices leave the range the int8
    codes cover: the extraction flags it, the int8 GEMM is skipped and the
    gated BF16 recomputation gives the BF16 path's result (non-finite where
    the reference's is)."""
    rng = np.random.RandomState(9)
    A, B = rng.randn(300, 4200), rng.randn(4200, 280)
    if side == "A row":
        A[17] *= scale
    else:
        B[:, 17] *= scale
    rho = O.compute_rho_f32(4200)
    if side == "A row":
        _, _, _, fail = s8_slices(A, rho, 4, 1, 1)
    else:
        _, _, _, fail = s8_slices(B, rho, 4, 1, 0)
    assert fail == 1
    C, _ = pipeline(A, B)
    assert same(C, bf16_pipeline(A, B, 4, 1))


@pytest.mark.parametrize("K", [64, 4200])
@pytest.mark.parametrize("scale", [2.0 ** -135, 2.0 ** 112])
def test_extreme_row_is_nan_like_the_reference(K, scale):
    """A row whose slices are non-finite in the reference's recurrence gives a
    NaN row there (matmul_numpy, pipeline='ondevice'); the fused accumulation
    must too, on the BF16 path (K = 64) and after the int8 fallback (K = 4200)."""
    import ozaki_jax_b200 as oz
    rng = np.random.RandomState(9)
    A, B = rng.randn(40, K), rng.randn(K, 30)
    A[17] *= scale
    with np.errstate(all="ignore"):
        R = O.ondevice_numpy(A, B, 4, 1)
    C = oz.matmul(A, B, pipeline="ondevice")
    assert np.array_equal(np.isnan(C), np.isnan(R))
    ok = ~np.isnan(R)
    assert O.rel_err(C[ok].reshape(-1, 30), R[ok].reshape(-1, 30)) <= 1e-12


def bf16_residual(A, X, Bv, n_hi, n_lo):
    """b - A X with fixed-point sums on BF16 slices (standalone entry points)."""
    rho = O.compute_rho_f32(A.shape[1])
    SA, k_pad, eA, _ = extract_device(torch.as_tensor(A).cuda(), rho, n_hi, n_lo, 1)
    SX, _, eX, _ = extract_device(torch.as_tensor(X).cuda(), rho, n_hi, n_lo, 0)
    return bf16_fixed_gemm(SA, eA, SX, eX, k_pad, A.shape[0], X.shape[1], rho, n_hi, n_lo,
                           alpha=-1.0, beta=1.0, Cin=torch.as_tensor(Bv).cuda())


def residual_pipeline(A, X, Bv, n_hi, n_lo):
    lib = L.load()
    N, K = A.shape
    M = X.shape[1]
    Ad, Xd, Bd = (torch.as_tensor(v).cuda() for v in (A, X, Bv))
    R = torch.full((N, M), float("nan"), dtype=torch.float64, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.check(lib.ozk_residual_f64(Ad.data_ptr(), K, Xd.data_ptr(), M, Bd.data_ptr(), M,
                                 R.data_ptr(), M, N, K, M, -1, n_hi, n_lo, None, 0, st.data_ptr(),
                                 stream()))
    torch.cuda.synchronize()
    return R.cpu().numpy(), int(st.item())


@pytest.mark.parametrize("N,K,M,n_hi,n_lo", [(1000, 5000, 16, 4, 1), (300, 4224, 5, 4, 1),
                                             (777, 6000, 1, 3, 1), (256, 8192, 16, 4, 2),
                                             (19200, 4224, 16, 4, 1)])
def test_skinny_s8_residual_matches_bf16(N, K, M, n_hi, n_lo):
    """Residuals (at most 16 right-hand sides) take the int8 all-pairs kernel;
    bit-identical to the BF16 narrow kernel's fixed-point result.  With fewer
    128-row tiles than SMs (the small cases), or 150 tiles on a 148-SM B200,
    each tile's K range is split over several CTAs and the int32 products
    added in a scratch before the fixed-point sums."""
    rng = np.random.RandomState(N + M)
    A = rng.randn(N, K) * np.exp(rng.randn(N, 1) * 2)
    X, Bv = rng.randn(K, M), rng.randn(N, M)
    R, st = residual_pipeline(A, X, Bv, n_hi, n_lo)
    assert st == 0
    assert same(R, bf16_residual(A, X, Bv, n_hi, n_lo))


@pytest.mark.parametrize("M", [16, 3])
def test_skinny_s8_matmul_matches_bf16(M):
    rng = np.random.RandomState(M)
    A, B = rng.randn(2000, 4500), rng.randn(4500, M)
    C, st = pipeline(A, B)
    assert st == 0
    assert same(C, bf16_pipeline(A, B, 4, 1))


def test_skinny_s8_falls_back_on_device():
    rng = np.random.RandomState(12)
    A, X, Bv = rng.randn(300, 4200), rng.randn(4200, 8), rng.randn(300, 8)
    A[5] *= 2.0 ** -135
    R, _ = residual_pipeline(A, X, Bv, 4, 1)
    assert same(R, bf16_residual(A, X, Bv, 4, 1))
    assert np.isnan(R[5]).all() and not np.isnan(np.delete(R, 5, axis=0)).any()
