"""Generate golden vectors by running the reference implementation itself.

Usage (in a container that has the reference source tree; JAX is not
needed):

    python tests/golden/make_golden.py [--ref /path/to/ozaki-jax]

The reference (Efithor/ozaki-jax v0.7.0) is pure Python + JAX.  A NumPy-backed
stand-in for `jax` (`tests/golden/refshim/jax`) lets its own functions run
unmodified; every FP32 step then executes as one IEEE round-to-nearest
NumPy operation.  Outputs (all small):

  golden_cases.npz   inputs, slices (as BF16 bit patterns), exponents and the
                     results of matmul / matmul_numpy / gram / residual per case
  golden_meta.json   rho table, pair schedules, preflight messages, reference
                     errors at 256x8192x256 (the 1.5x accuracy gates)

The GPU box never runs this script; tests read the committed files.
"""

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _bf16_bits(x32):
    """FP32 array holding BF16-exact values -> uint16 BF16 bit patterns."""
    b = np.ascontiguousarray(x32, dtype=np.float32).view(np.uint32)
    assert np.all((b & 0xFFFF) == 0), "slice value is not BF16-exact"
    return (b >> 16).astype(np.uint16)


def cases():
    """Seeded inputs (name -> (A, B)).  Draw order is documented per case."""
    out = {}
    rng = np.random.RandomState(0)          # CI case: A then B, 64x64 N(0,1)
    out["n64_s0"] = (rng.randn(64, 64), rng.randn(64, 64))
    rng = np.random.RandomState(1)          # ragged shapes
    out["rect_37x100x23"] = (rng.randn(37, 100), rng.randn(100, 23))
    rng = np.random.RandomState(2)          # zero rows / columns and signed zeros
    A = rng.randn(24, 48)
    B = rng.randn(48, 16)
    A[3] = 0.0
    A[7] = -0.0
    A[9, ::2] = -0.0
    B[:, 5] = 0.0
    B[::3, 6] = -0.0
    out["zeros_24x48x16"] = (A, B)
    rng = np.random.RandomState(3)          # wide dynamic range, phi = 10
    A = (rng.rand(40, 96) - 0.5) * np.exp(10 * rng.randn(40, 96))
    B = (rng.rand(96, 32) - 0.5) * np.exp(10 * rng.randn(96, 32))
    out["wide_phi10_40x96x32"] = (A, B)
    rng = np.random.RandomState(4)          # K = 1040 -> rho = 18
    out["k1040_8x1040x8"] = (rng.randn(8, 1040), rng.randn(1040, 8))
    rng = np.random.RandomState(5)          # tiny and huge row/column scales
    A = rng.randn(16, 32)
    B = rng.randn(32, 12)
    A[0] *= 2.0 ** -120
    A[1] *= 2.0 ** 100
    A[2] *= 2.0 ** -140
    B[:, 0] *= 2.0 ** -110
    B[:, 1] *= 2.0 ** 90
    out["scales_16x32x12"] = (A, B)
    rng = np.random.RandomState(6)          # maxima in the log2 round-up zone
    A = rng.rand(12, 20) * 0.5
    B = rng.rand(20, 10) * 0.5
    tops = [np.float32(16.0), np.float32(2.0 ** 30), np.float32(2.0 ** -20),
            np.float32(2.0 ** 100), np.float32(2.0 ** -100), np.float32(1.0)]
    for i, t in enumerate(tops):
        A[i, i] = float(np.nextafter(t, np.float32(0)))          # one ulp below
        A[i + 6, i] = float(np.float32(t) * np.float32(1 - 2.0 ** -22))
        B[i, i] = float(np.nextafter(t, np.float32(0)))
    out["log2_edges_12x20x10"] = (A, B)
    rng = np.random.RandomState(7)          # degenerate shapes
    out["vec_1x128x1"] = (rng.randn(1, 128), rng.randn(128, 1))
    out["outer_48x1x40"] = (rng.randn(48, 1), rng.randn(1, 40))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("OZAKI_REF"),
                    help="checkout of the reference project (or set OZAKI_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref or set OZAKI_REF to the reference checkout")
    sys.path.insert(0, os.path.join(HERE, "refshim"))
    sys.path.insert(0, args.ref)
    import importlib

    import ozaki_jax as oj
    ex = importlib.import_module("ozaki_jax.extract")
    mm = importlib.import_module("ozaki_jax.matmul")
    pga = importlib.import_module("ozaki_jax.pallas_gemm_accum")

    arrays = {}
    meta = {"reference_version": oj.__version__, "cases": {}}
    presets = {"high": (4, 1), "medium": (3, 1), "max": (5, 4), "c42": (4, 2)}
    for name, (A, B) in cases().items():
        info = {"shape": [A.shape[0], A.shape[1], B.shape[1]]}
        arrays[f"{name}/A"] = A
        arrays[f"{name}/B"] = B
        K = A.shape[1]
        rho = ex._compute_rho_f32(K)
        info["rho"] = rho
        A_hi, A_lo = mm._double_f32_split(A)
        B_hi, B_lo = mm._double_f32_split(B)
        for part, X in (("A_hi", A_hi), ("A_lo", A_lo)):
            s, e = ex.f32_extract_split_rows(X, rho, 5)
            arrays[f"{name}/{part}/slices"] = np.stack([_bf16_bits(v) for v in s])
            arrays[f"{name}/{part}/exps"] = np.stack(e).astype(np.int16)
        for part, X in (("B_hi", B_hi), ("B_lo", B_lo)):
            s, e = ex.f32_extract_split_cols(X, rho, 5)
            arrays[f"{name}/{part}/slices"] = np.stack([_bf16_bits(v) for v in s])
            arrays[f"{name}/{part}/exps"] = np.stack(e).astype(np.int16)
        full = name in ("n64_s0", "rect_37x100x23")
        for pname, prec in presets.items():
            if not full and pname in ("medium", "c42"):
                continue
            n_hi, n_lo = prec
            bgs = (tuple([n_hi] * n_hi), tuple([n_lo] * n_hi), tuple([n_hi] * n_lo))
            ch, cl = mm._fully_fused_ondevice_jit(A, B, rho, n_hi, n_lo, bgs)
            arrays[f"{name}/{pname}/C_hi"] = np.asarray(ch, dtype=np.float32)
            arrays[f"{name}/{pname}/C_lo"] = np.asarray(cl, dtype=np.float32)
            arrays[f"{name}/{pname}/fused"] = oj.matmul(
                A, B, pipeline="ondevice", accumulation="fused", precision=prec)
            il = oj.matmul(A, B, pipeline="ondevice", accumulation="bf16_interleaved",
                           precision=prec)
            assert np.array_equal(il, arrays[f"{name}/{pname}/fused"], equal_nan=True)
            arrays[f"{name}/{pname}/numpy"] = oj.matmul_numpy(
                A, B, pipeline="ondevice", precision=prec)
        try:
            arrays[f"{name}/host8"] = oj.matmul_numpy(A, B)
        except ValueError as e:
            info["host8_error"] = str(e)
        meta["cases"][name] = info

    # gram and residual (mode='ozaki') on small seeded inputs
    rng = np.random.RandomState(42)
    G_A = rng.randn(96, 40) * (10.0 ** (-6 * np.arange(40) / 39))[None, :]
    arrays["gram/A"] = G_A
    for pname in ("high", "medium"):
        for acc in ("bf16_interleaved", "fused"):
            arrays[f"gram/{pname}/{acc}"] = oj.gram(G_A, mode="ozaki", precision=pname,
                                                    accumulation=acc)
    rng = np.random.RandomState(43)
    R_A = rng.randn(64, 64) + 64 * np.eye(64)
    R_x = rng.randn(64, 4)
    R_b = rng.randn(64, 4)
    R_xv = rng.randn(64)
    R_bv = rng.randn(64)
    for k, v in (("A", R_A), ("x", R_x), ("b", R_b), ("xv", R_xv), ("bv", R_bv)):
        arrays[f"residual/{k}"] = v
    for pname in ("high", "medium"):
        for acc in ("bf16_interleaved", "fused"):
            arrays[f"residual/{pname}/{acc}"] = oj.residual(
                R_A, R_x, R_b, mode="ozaki", precision=pname, accumulation=acc)
    arrays["residual/high/vec"] = oj.residual(R_A, R_xv, R_bv, mode="ozaki")

    # policies
    meta["rho_f32"] = {str(K): ex._compute_rho_f32(K) for K in
                       (0, 1, 2, 64, 1000, 1024, 1025, 1040, 2048, 4096, 4097, 8192,
                        8193, 16384, 32768, 65536, 10 ** 6, 2 ** 23, 2 ** 23 + 1)}
    meta["rho_f64"] = {str(K): ex._compute_rho(K) for K in
                       (1, 2, 64, 256, 1024, 4096, 8192, 10000, 65536)}
    meta["pair_schedule"] = {}
    for n_hi, n_lo in ((4, 1), (3, 1), (5, 4), (4, 2), (1, 1), (2, 3)):
        pa, pb, npairs, groups, bounds = pga._make_pair_schedule(n_hi, n_lo)
        meta["pair_schedule"][f"{n_hi},{n_lo}"] = {
            "pair_a": list(pa), "pair_b": list(pb), "n_pairs": npairs,
            "groups": [[a, list(ps)] for a, ps in groups], "bounds": list(bounds)}

    # preflight messages (matmul.py:119-135, :600-638)
    msgs = {}
    rng = np.random.RandomState(9)
    for label, kw, A, B in (
            ("ondevice_nan", dict(pipeline="ondevice"), np.full((4, 4), np.nan), np.ones((4, 4))),
            ("ondevice_inf", dict(pipeline="ondevice"), np.ones((4, 4)), np.full((4, 4), np.inf)),
            ("host_k10000", dict(pipeline="host"), rng.randn(2, 10000), rng.randn(10000, 2)),
            ("bad_precision", dict(pipeline="ondevice", precision="invalid"), np.ones((2, 2)), np.ones((2, 2))),
            ("bad_tuple", dict(pipeline="ondevice", precision=(0, 1)), np.ones((2, 2)), np.ones((2, 2))),
            ("bad_accumulation", dict(pipeline="ondevice", accumulation="x"), np.ones((2, 2)), np.ones((2, 2))),
            ("bad_pipeline", dict(pipeline="gpu"), np.ones((2, 2)), np.ones((2, 2))),
            ("bad_safe_mode", dict(pipeline="ondevice", safe_mode="ignore"), np.ones((2, 2)), np.ones((2, 2))),
            ("bad_shapes", dict(pipeline="ondevice"), np.ones((2, 3)), np.ones((2, 2))),
            ("bad_rank", dict(pipeline="ondevice"), np.ones(3), np.ones((3, 2)))):
        try:
            oj.matmul(A, B, **kw)
            msgs[label] = None
        except ValueError as e:
            msgs[label] = str(e)
    # gram / residual argument checks (gram.py:66-84, solve.py:56-75, :113-128)
    one = np.ones
    for label, fn, args, kw in (
            ("gram_bad_mode", oj.gram, (one((4, 4)),), dict(mode="invalid")),
            ("gram_bad_accumulation", oj.gram, (one((4, 4)),), dict(mode="ozaki", accumulation="host")),
            ("gram_not_2d", oj.gram, (one(4),), dict(mode="ozaki")),
            ("residual_bad_mode", oj.residual, (one((3, 4)), one(4), one(3)), dict(mode="invalid")),
            ("residual_bad_accumulation", oj.residual, (one((3, 4)), one(4), one(3)),
             dict(mode="ozaki", accumulation="host")),
            ("residual_not_2d", oj.residual, (one(4), one(4), one(4)), dict(mode="ozaki")),
            ("residual_x_length", oj.residual, (one((3, 4)), one(5), one(3)), dict(mode="ozaki")),
            ("residual_b_vector", oj.residual, (one((3, 4)), one(4), one(4)), dict(mode="ozaki")),
            ("residual_x_rows", oj.residual, (one((3, 4)), one((5, 2)), one((3, 2))), dict(mode="ozaki")),
            ("residual_b_matrix", oj.residual, (one((3, 4)), one((4, 2)), one((3, 3))), dict(mode="ozaki")),
            ("residual_x_ndim", oj.residual, (one((3, 4)), one((4, 1, 1)), one(3)), dict(mode="ozaki"))):
        try:
            fn(*args, **kw)
            msgs[label] = None
        except ValueError as e:
            msgs[label] = str(e)
    meta["messages"] = msgs
    fb_A, fb_B = rng.randn(2, 10000), rng.randn(10000, 2)
    arrays["fallback/A"], arrays["fallback/B"] = fb_A, fb_B
    arrays["fallback/C"] = oj.matmul(fb_A, fb_B, pipeline="host", safe_mode="fallback")

    # reference errors at 256 x 8192 x 256, N(0,1), RandomState(0), A then B:
    # these set the 1.5x accuracy gates used on the GPU.
    rng = np.random.RandomState(0)
    A = rng.randn(256, 8192)
    B = rng.randn(8192, 256)
    R = A @ B
    errs = {}
    for pname in ("high", "medium", "max"):
        Cf = oj.matmul(A, B, pipeline="ondevice", accumulation="fused", precision=pname)
        Cn = oj.matmul_numpy(A, B, pipeline="ondevice", precision=pname)
        errs[pname] = {"fused": float(np.linalg.norm(Cf - R) / np.linalg.norm(R)),
                       "numpy": float(np.linalg.norm(Cn - R) / np.linalg.norm(R))}
    meta["ref_err_256x8192x256"] = errs

    np.savez_compressed(os.path.join(HERE, "golden_cases.npz"), **arrays)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main()
