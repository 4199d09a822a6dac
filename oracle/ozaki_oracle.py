"""CPU oracle for the Ozaki matmul path -- TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy, the arithmetic of the reference
implementation (Efithor/ozaki-jax v0.7.0, package `ozaki_jax`) for the
on-device matmul path and the callers around it.  Each function names the
reference lines it follows.  It is the checker the GPU results are compared
with; it is imported only by `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py`.  The product path
(`ozaki_jax_b200`) never imports it and has no CPU fallback.

Parity pins: `tests/test_oracle.py` checks every function here against
golden vectors produced by running the reference's own code
(`tests/golden/make_golden.py`, a NumPy-backed stand-in for `jax`), bit for
bit where the reference is deterministic (slices, exponents, products,
2Sum (C_hi, C_lo)), and exactly for the FP64 accumulations.

Arithmetic conventions: every FP32 step is written as a separate NumPy
float32 operation, i.e. one IEEE round-to-nearest-even op, which is what the
reference's traced FP32 programs express.
"""

import math

import numpy as np

F32 = np.float32
F64 = np.float64

# ---------------------------------------------------------------------------
# Policies: rho, presets, pair schedules
# ---------------------------------------------------------------------------

PRESETS = {"high": (4, 1), "medium": (3, 1), "max": (5, 4)}  # matmul.py:168-172


def compute_rho_f32(K):
    """rho for FP32 extraction (extract.py:109-113): max(ceil(24-(24-ceil(log2 max(K,2)))/2), 17)."""
    lg = math.ceil(math.log2(max(K, 2)))
    return max(int(math.ceil(24 - (24 - lg) / 2)), 17)


def compute_rho_f64(K):
    """rho for the FP64 host pipeline (extract.py:12-18): max(ceil(53-(24-ceil(log2 max(K,2)))/2), 46)."""
    lg = math.ceil(math.log2(max(K, 2)))
    return max(int(math.ceil(53 - (24 - lg) / 2)), 46)


def resolve_precision(precision):
    """Preset name or (n_hi, n_lo) tuple -> (n_hi, n_lo) (matmul.py:175-194)."""
    if isinstance(precision, tuple) and len(precision) == 2:
        n_hi, n_lo = precision
        if n_hi < 1 or n_lo < 1:
            raise ValueError("custom precision needs n_hi >= 1 and n_lo >= 1")
        return precision
    if precision not in PRESETS:
        raise ValueError(f"unknown precision {precision!r}")
    return PRESETS[precision]


def ondevice_pairs(n_hi, n_lo):
    """Slice-pair order of the on-device pipeline (pallas_gemm_accum.py:26-87).

    Slices are indexed hi first (0..n_hi-1) then lo (n_hi..n_hi+n_lo-1) on
    both sides.  Order: hi x hi (row-major), hi x lo, lo x hi; lo x lo is
    never formed.  Returns (pairs, groups, block_bounds) where groups[g] =
    (a_slice, [pair indices]) and block_bounds are cumulative group counts
    of the three blocks.
    """
    pairs, groups = [], []
    for i in range(n_hi):
        groups.append((i, list(range(len(pairs), len(pairs) + n_hi))))
        pairs += [(i, j) for j in range(n_hi)]
    for i in range(n_hi):
        groups.append((i, list(range(len(pairs), len(pairs) + n_lo))))
        pairs += [(i, n_hi + j) for j in range(n_lo)]
    for i in range(n_lo):
        groups.append((n_hi + i, list(range(len(pairs), len(pairs) + n_hi))))
        pairs += [(n_hi + i, j) for j in range(n_hi)]
    return pairs, groups, (n_hi, 2 * n_hi, 2 * n_hi + n_lo)


def triangular_pairs(n_slices):
    """Host-pipeline pairs i + j <= n-1, i outer (matmul.py:23-32, :54-60)."""
    return [(i, j) for i in range(n_slices) for j in range(n_slices) if i + j <= n_slices - 1]


# ---------------------------------------------------------------------------
# Splitting and extraction
# ---------------------------------------------------------------------------

def double_f32_split(X):
    """hi = RN32(x), lo = RN32(x - hi) (matmul.py:197-201)."""
    X = np.asarray(X, dtype=F64)
    with np.errstate(over="ignore", invalid="ignore"):
        hi = X.astype(F32)
        lo = (X - hi.astype(F64)).astype(F32)
    return hi, lo


def floor_log2_f32(m):
    """floor(RN32(log2(m))) for positive FP32 m, the reference's exponent rule
    (extract.py:130, :171).  Near the top of a binade the rounded log2 reaches
    the next integer, so this is not the IEEE exponent there."""
    with np.errstate(divide="ignore"):
        return np.floor(np.log2(np.asarray(m, dtype=F32)).astype(F32))


def _pow2_f32(n):
    """ldexp(1.0f, n) in FP32, overflow to inf / underflow to 0 like NumPy."""
    with np.errstate(over="ignore", under="ignore"):
        return np.ldexp(np.ones(np.shape(n), dtype=F32), np.asarray(n).astype(np.int32))


def _extract_f32(X32, rho, n_slices, axis):
    """Sigma-trick extraction along `axis` (1 = per row, 0 = per column).

    Per slice (extract.py:124-152 rows, :165-189 columns):
      m = max|r| along the line; c = floor(RN32 log2 m), 0 for an all-zero line;
      sigma = RN32(0.75 * 2^(rho+c)); v = RN32(RN32(r+sigma)-sigma), 0 on zero lines;
      r = RN32(r - v); slice = RN32(v * 2^-c); exponent = c.
    Returns (list of FP32 slices, list of FP32 exponent vectors).
    """
    r = np.array(X32, dtype=F32, copy=True)
    slices, exps = [], []
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        for _ in range(n_slices):
            m = np.max(np.abs(r), axis=axis).astype(F32)
            zero = m == 0
            c = floor_log2_f32(np.where(zero, F32(1.0), m))
            c = np.where(zero, F32(0.0), c).astype(F32)
            sigma = (F32(0.75) * _pow2_f32(rho + c)).astype(F32)
            sig = sigma[:, None] if axis == 1 else sigma[None, :]
            zmask = zero[:, None] if axis == 1 else zero[None, :]
            v = ((r + sig).astype(F32) - sig).astype(F32)
            v = np.where(zmask, F32(0.0), v).astype(F32)
            r = (r - v).astype(F32)
            inv = _pow2_f32(-c)
            inv = inv[:, None] if axis == 1 else inv[None, :]
            slices.append((v * inv).astype(F32))
            exps.append(c)
    return slices, exps


def extract_rows_f32(X32, rho, n_slices):
    """f32_extract_split_rows (extract.py:116-154)."""
    return _extract_f32(X32, rho, n_slices, axis=1)


def extract_cols_f32(X32, rho, n_slices):
    """f32_extract_split_cols (extract.py:157-191)."""
    return _extract_f32(X32, rho, n_slices, axis=0)


def _extract_f64(X, rho, n_slices, axis):
    """FP64 sigma-trick extraction for the host pipeline (extract.py:21-103).

    Same recurrence in FP64 with floor(log2) in FP64; slices are rounded to
    FP32 storage after normalisation by 2^-c.
    """
    r = np.array(X, dtype=F64, copy=True)
    slices, exps = [], []
    with np.errstate(over="ignore", invalid="ignore", under="ignore", divide="ignore"):
        for _ in range(n_slices):
            m = np.max(np.abs(r), axis=axis)
            zero = m == 0
            c = np.floor(np.log2(np.where(zero, 1.0, m)))
            c = np.where(zero, 0.0, c)
            sigma = 0.75 * np.ldexp(np.ones(c.shape, F64), (rho + c).astype(np.int64))
            sig = sigma[:, None] if axis == 1 else sigma[None, :]
            zmask = zero[:, None] if axis == 1 else zero[None, :]
            v = (r + sig) - sig
            v = np.where(zmask, 0.0, v)
            r = r - v
            inv = np.ldexp(np.ones(c.shape, F64), (-c).astype(np.int64))
            inv = inv[:, None] if axis == 1 else inv[None, :]
            slices.append((v * inv).astype(F32))
            exps.append(c)
    return slices, exps


def extract_rows_f64(X, rho, n_slices):
    """extract_split_rows (extract.py:21-65)."""
    return _extract_f64(X, rho, n_slices, axis=1)


def extract_cols_f64(X, rho, n_slices):
    """extract_split_cols (extract.py:68-103)."""
    return _extract_f64(X, rho, n_slices, axis=0)


def extract_ondevice(A, B, n_hi, n_lo, rho=None):
    """Split + extract both operands of the on-device pipeline.

    Returns (SA, eA, SB, eB, rho): SA (n_hi+n_lo, N, K) FP32 slices of A
    (hi slices first), eA (n_hi+n_lo, N) exponents, SB (n_hi+n_lo, K, M)
    and eB (n_hi+n_lo, M) for B (matmul.py:746-750).
    """
    A = np.asarray(A, dtype=F64)
    B = np.asarray(B, dtype=F64)
    if rho is None:
        rho = compute_rho_f32(A.shape[1])
    A_hi, A_lo = double_f32_split(A)
    B_hi, B_lo = double_f32_split(B)
    ah, eah = extract_rows_f32(A_hi, rho, n_hi)
    al, eal = extract_rows_f32(A_lo, rho, n_lo)
    bh, ebh = extract_cols_f32(B_hi, rho, n_hi)
    bl, ebl = extract_cols_f32(B_lo, rho, n_lo)
    SA = np.stack(ah + al)
    SB = np.stack(bh + bl)
    return SA, np.stack(eah + eal), SB, np.stack(ebh + ebl), rho


# ---------------------------------------------------------------------------
# Products and accumulation
# ---------------------------------------------------------------------------

def slice_products(SA, SB, pairs):
    """P_p = SA[a] @ SB[b] in FP32 (matmul.py:753-774).  Exact by construction:
    every partial sum is an integer multiple of the slice grid below 2^24."""
    return np.stack([(SA[a].astype(F32) @ SB[b].astype(F32)).astype(F32) for a, b in pairs])


def accumulate_block_products(P, eA, eB, n_hi, n_lo):
    """FP64 accumulation of the on-device pipeline's NumPy mirror
    (matmul.py:543-597): per group, FP32 column scaling, FP64 inner sum,
    FP64 row scaling, FP64 add into C."""
    pairs, groups, _ = ondevice_pairs(n_hi, n_lo)
    N, M = P.shape[1], P.shape[2]
    C = np.zeros((N, M), dtype=F64)
    for a, pidx in groups:
        inner = np.zeros((N, M), dtype=F64)
        for p in pidx:
            col = _pow2_f32(eB[pairs[p][1]])
            inner += (P[p] * col[None, :]).astype(F32)
        inner *= np.ldexp(np.ones(N, F64), eA[a].astype(np.int64))[:, None]
        C += inner
    return C


def accumulation_scales(eA, eB, n_hi, n_lo):
    """Per-product FP32 column scales and per-group FP32 row scales
    (pallas_ops.py:107-175, matmul.py:264-277)."""
    pairs, groups, bounds = ondevice_pairs(n_hi, n_lo)
    col = np.stack([_pow2_f32(eB[b]) for _, b in pairs])
    row = np.stack([_pow2_f32(eA[a]) for a, _ in groups])
    sizes = []
    prev = 0
    for end in bounds:
        sizes.append(tuple(len(groups[g][1]) for g in range(prev, end)))
        prev = end
    return col, row, tuple(sizes)


def _twosum(s_hi, s_lo, x):
    """2Sum of x into (s_hi, s_lo) in FP32 (pallas_ops.py:195-199)."""
    t = (s_hi + x).astype(F32)
    e = ((s_hi - t).astype(F32) + x).astype(F32)
    return t, (s_lo + e).astype(F32)


def accumulate_2sum(P, col_scales, row_scales, block_group_sizes):
    """Scaled FP32 2Sum accumulation (pallas_ops.py:178-239).

    Per group: inner 2Sum over the group's products scaled by their column
    scale; both inner words times the group's row scale; 2Sum of inner_hi
    then inner_lo into the block.  Then the block hi words are 2Summed in
    block order, followed by the block lo words.  Returns (C_hi, C_lo).
    """
    N, M = P.shape[1], P.shape[2]
    z = lambda: np.zeros((N, M), dtype=F32)  # noqa: E731
    blocks = []
    p = g = 0
    with np.errstate(over="ignore", invalid="ignore"):
        for sizes in block_group_sizes:
            bh, bl = z(), z()
            for gs in sizes:
                ih, il = z(), z()
                for _ in range(gs):
                    ih, il = _twosum(ih, il, (P[p] * col_scales[p][None, :]).astype(F32))
                    p += 1
                rs = row_scales[g][:, None]
                ih, il = (ih * rs).astype(F32), (il * rs).astype(F32)
                bh, bl = _twosum(bh, bl, ih)
                bh, bl = _twosum(bh, bl, il)
                g += 1
            blocks.append((bh, bl))
        ch, cl = z(), z()
        for bh, _ in blocks:
            ch, cl = _twosum(ch, cl, bh)
        for _, bl in blocks:
            ch, cl = _twosum(ch, cl, bl)
    return ch, cl


# ---------------------------------------------------------------------------
# Pipelines
# ---------------------------------------------------------------------------

def ondevice_numpy(A, B, n_hi=4, n_lo=1):
    """matmul_numpy(pipeline='ondevice') without the preflight
    (matmul.py:731-778): extraction, exact FP32 products, FP64 accumulation."""
    SA, eA, SB, eB, _ = extract_ondevice(A, B, n_hi, n_lo)
    pairs, _, _ = ondevice_pairs(n_hi, n_lo)
    return accumulate_block_products(slice_products(SA, SB, pairs), eA, eB, n_hi, n_lo)


def fused_ondevice(A, B, n_hi=4, n_lo=1, rho=None):
    """The reference's fused / bf16_interleaved / ondevice accumulation result
    (matmul.py:236-281 + pallas_ops.py:178-239, :514-526): returns
    (C_hi, C_lo, C = f64(C_hi) + f64(C_lo))."""
    SA, eA, SB, eB, _ = extract_ondevice(A, B, n_hi, n_lo, rho)
    pairs, _, _ = ondevice_pairs(n_hi, n_lo)
    P = slice_products(SA, SB, pairs)
    col, row, bgs = accumulation_scales(eA, eB, n_hi, n_lo)
    ch, cl = accumulate_2sum(P, col, row, bgs)
    return ch, cl, ch.astype(F64) + cl.astype(F64)


def host_numpy(A, B, n_slices=8):
    """matmul_numpy(pipeline='host') without the preflight (matmul.py:881-900):
    FP64 extraction, triangular pairs, FP32 products rescaled in FP64."""
    A = np.asarray(A, dtype=F64)
    B = np.asarray(B, dtype=F64)
    rho = compute_rho_f64(A.shape[1])
    SA, eA = extract_rows_f64(A, rho, n_slices)
    SB, eB = extract_cols_f64(B, rho, n_slices)
    C = np.zeros((A.shape[0], B.shape[1]), dtype=F64)
    for i, j in triangular_pairs(n_slices):
        P = (SA[i] @ SB[j]).astype(F32).astype(F64)
        P *= np.ldexp(np.ones(A.shape[0], F64), eA[i].astype(np.int64))[:, None]
        P *= np.ldexp(np.ones(B.shape[1], F64), eB[j].astype(np.int64))[None, :]
        C += P
    return C


def gram_ozaki(A, n_hi=4, n_lo=1):
    """gram(mode='ozaki') (gram.py:19-37, :92-95): ozaki(A^T, A) with rho from
    the row count, then (G + G^T) / 2.  bf16_interleaved and fused agree."""
    A = np.asarray(A, dtype=F64)
    rho = compute_rho_f32(A.shape[0])
    _, _, G = fused_ondevice(A.T, A, n_hi, n_lo, rho)
    return (G + G.T) * 0.5


def residual_ozaki(A, x, b, n_hi=4, n_lo=1):
    """residual(mode='ozaki') (solve.py:38-53, :78-82, :131-150): b - ozaki(A, x),
    a vector x taken as one column."""
    A = np.asarray(A, dtype=F64)
    x = np.asarray(x, dtype=F64)
    b = np.asarray(b, dtype=F64)
    vec = x.ndim == 1
    X = x[:, None] if vec else x
    Bv = b[:, None] if vec else b
    rho = compute_rho_f32(A.shape[1])
    _, _, AX = fused_ondevice(A, X, n_hi, n_lo, rho)
    r = Bv - AX
    return r[:, 0] if vec else r


# ---------------------------------------------------------------------------
# Preflight (safety reports) and the exact reference product
# ---------------------------------------------------------------------------

def ondevice_safety_report(A, B, n_hi, n_lo):
    """_ondevice_safety_report (matmul.py:600-638), reasons with the same text."""
    K = A.shape[1]
    rho = compute_rho_f32(K)
    bits = 24 - rho
    reasons = []
    if bits <= 0:
        reasons.append(f"non-positive bits per slice ({bits}); K={K} is too "
                       "large for FP32 extraction")
    else:
        if K * (2 ** bits - 1) ** 2 >= 2 ** 24:
            reasons.append(f"K={K} violates BF16->FP32 exact inner-product bound "
                           f"(need K <= {int(2 ** 24 / (2 ** bits - 1) ** 2)})")
    if not np.isfinite(A).all() or not np.isfinite(B).all():
        reasons.append("inputs contain NaN or Inf")
    return {"safe": not reasons, "rho": rho, "bits_per_slice": bits, "n_hi": n_hi,
            "n_lo": n_lo, "n_gemms": n_hi * n_hi + 2 * n_hi * n_lo, "reasons": reasons}


def host_safety_report(A, B, n_slices):
    """_ozaki_safety_report (matmul.py:77-116)."""
    K = A.shape[1]
    rho = compute_rho_f64(K)
    bits = 53 - rho
    reasons = []
    if bits <= 0:
        reasons.append(f"non-positive bits per slice ({bits}); K={K} is too large "
                       "for this BF16->FP32 exactness model")
    elif K * (2 ** bits - 1) ** 2 >= 2 ** 24:
        reasons.append(f"K={K} violates BF16->FP32 exact inner-product bound "
                       f"(need K <= {int(2 ** 24 / (2 ** bits - 1) ** 2)})")
    if n_slices * max(bits, 0) < 53:
        reasons.append(f"insufficient slice budget: n_slices*bits_per_slice="
                       f"{n_slices * max(bits, 0)} < 53")
    if not np.isfinite(A).all() or not np.isfinite(B).all():
        reasons.append("inputs contain NaN or Inf")
    return {"safe": not reasons, "rho": rho, "bits_per_slice": bits, "reasons": reasons}


def exact_product(A, B):
    """Correctly rounded FP64 A @ B for small operands (the error reference).

    Each operand is split error-free, per row of A and per column of B, into
    FP64 pieces of at most 18 significant bits on a common grid (the FP64
    sigma trick with rho = 36), until nothing is left.  Every piece product
    and its K-sum is then exact in FP64 (36 bits + log2 K <= 53 for
    K <= 2^17), and the exact partial matrices are summed per element with
    math.fsum, which rounds the exact sum once.
    """
    A = np.asarray(A, dtype=F64)
    B = np.asarray(B, dtype=F64)
    assert A.shape[1] <= 2 ** 17

    def pieces(X, axis):
        r = X.copy()
        out = []
        while np.any(r != 0):
            assert len(out) < 200
            m = np.max(np.abs(r), axis=axis)
            zero = m == 0
            c = np.where(zero, 0.0, np.floor(np.log2(np.where(zero, 1.0, m))))
            sigma = 0.75 * np.ldexp(np.ones(c.shape), (c + 36).astype(np.int64))
            sig = sigma[:, None] if axis == 1 else sigma[None, :]
            v = (r + sig) - sig
            v = np.where((zero[:, None] if axis == 1 else zero[None, :]), 0.0, v)
            r = r - v
            out.append(v)
        return out or [np.zeros_like(X)]

    PA, PB = pieces(A, 1), pieces(B, 0)
    N, M = A.shape[0], B.shape[1]
    stack = np.stack([a @ b for a in PA for b in PB]).reshape(len(PA) * len(PB), -1)
    out = np.array([math.fsum(stack[:, i]) for i in range(N * M)], dtype=F64)
    return out.reshape(N, M)


def rel_err(C, R):
    """Normwise relative error ||C-R||_F / ||R||_F, scaled by max|R| first to
    avoid overflow (benchmarks/ci_cpu_validate.py:13-19, stress_test.py:24-37)."""
    C = np.asarray(C, dtype=F64)
    R = np.asarray(R, dtype=F64)
    s = np.max(np.abs(R)) if R.size else 0.0
    if not np.isfinite(s) or s == 0:
        s = 1.0
    d = np.linalg.norm((R / s).ravel())
    if d == 0:
        d = np.linalg.norm((C / s).ravel())
    if d == 0:
        return 0.0
    return float(np.linalg.norm(((C - R) / s).ravel()) / d)
