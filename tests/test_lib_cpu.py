"""CPU-only checks of the boundary: the C-ABI library loads, exports every
symbol the header declares, and its host-side policies match the reference."""

import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "ozaki_b200.h")


def header_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ozk_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # every binding in the Python layer is declared in the header
    assert set(_lib.SIGNATURES) <= set(names)


def test_version_and_strerror():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    assert b"sm_100a" in lib.ozk_version()
    for code in range(-8, 1):
        assert lib.ozk_strerror(code)


def test_rho_policy_matches_reference(golden):
    from ozaki_jax_b200 import _lib
    _, meta = golden
    lib = _lib.load()
    for K, rho in meta["rho_f32"].items():
        assert lib.ozk_compute_rho_f32(int(K)) == rho, K
    for K, rho in meta["rho_f64"].items():
        assert lib.ozk_compute_rho_f64(int(K)) == rho, K


def test_pair_schedule_matches_reference(golden):
    from ozaki_jax_b200 import _lib
    _, meta = golden
    lib = _lib.load()
    for key, ref in meta["pair_schedule"].items():
        n_hi, n_lo = map(int, key.split(","))
        pa = (ctypes.c_uint8 * 256)()
        pb = (ctypes.c_uint8 * 256)()
        n = lib.ozk_pair_schedule(n_hi, n_lo, pa, pb, 256)
        assert n == ref["n_pairs"]
        assert list(pa[:n]) == ref["pair_a"] and list(pb[:n]) == ref["pair_b"]
    pa = (ctypes.c_uint8 * 256)()
    pb = (ctypes.c_uint8 * 256)()
    n = lib.ozk_triangular_schedule(8, pa, pb, 256)
    assert n == 36
    assert [(a, b) for a, b in zip(pa[:n], pb[:n])] == \
        [(i, j) for i in range(8) for j in range(8) if i + j <= 7]


def test_argument_errors_return_codes():
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    # NULL pointers and bad shapes are refused before any device work
    assert lib.ozk_matmul_f64(None, 1, None, 1, None, 1, 1, 1, 1, -1, 4, 1, 0, None, 0, None,
                              None) == _lib.OZK_ERR_ARG
    assert lib.ozk_pair_schedule(0, 1, None, None, 0) == _lib.OZK_ERR_ARG
    assert lib.ozk_slice_gemm(None, None, 1, None, None, 1, 1, 1, 64, None, None, 1, 0, 0, 1.0,
                              0.0, None, 0, None, 0, None, None, 0, 0, None, None) == _lib.OZK_ERR_ARG
    assert "NULL" in _lib.detail()


def test_every_entry_point_checks_arguments_before_device_work():
    """Each compute entry point refuses bad arguments with its status code
    (never an exception, never a device call): NULL pointers, shapes, leading
    dimensions, presets, the exact-product bound, workspace limits.  Empty
    products return OZK_OK without touching the device."""
    from ozaki_jax_b200 import _lib
    lib = _lib.load()
    ARG, UNSAFE, WS, OK = _lib.OZK_ERR_ARG, _lib.OZK_ERR_UNSAFE, _lib.OZK_ERR_WORKSPACE, _lib.OZK_OK
    buf = (ctypes.c_double * 16)()
    p = ctypes.addressof(buf)  # a host address: never dereferenced by these calls
    big = 2 ** 23              # K beyond the FP32 extraction's exact-product bound
    # matmul: shapes, leading dimensions, accumulation mode, preset, bound, empty
    mm = lib.ozk_matmul_f64
    assert mm(p, 4, p, 4, p, 4, 4, 0, 4, -1, 4, 1, 2, None, 0, None, None) == ARG
    assert mm(p, 3, p, 4, p, 4, 4, 4, 4, -1, 4, 1, 2, None, 0, None, None) == ARG
    assert mm(p, 4, p, 4, p, 4, 4, 4, 4, -1, 4, 1, 7, None, 0, None, None) == ARG
    assert mm(p, 4, p, 4, p, 4, 4, 4, 4, -1, 0, 1, 2, None, 0, None, None) == ARG
    assert mm(p, big, p, 4, p, 4, 4, big, 4, -1, 4, 1, 2, None, 0, None, None) == UNSAFE
    assert mm(p, 4, p, 4, p, 4, 0, 4, 4, -1, 4, 1, 2, None, 0, None, None) == OK
    # host-buffer matmul
    hb = lib.ozk_matmul_f64_hostbuf
    flags = ctypes.c_int32(0)
    assert hb(None, 4, p, 4, p, 4, 4, 4, 4, -1, 4, 1, 2, 0, None, 0, ctypes.byref(flags),
              None) == ARG
    assert hb(p, 4, p, 4, p, 4, 4, 4, 4, -1, 4, 1, 9, 0, None, 0, ctypes.byref(flags),
              None) == ARG
    # allocation-free matmul: presets and its fixed scratch limit
    na = lib.ozk_matmul_f64_noalloc
    assert na(p, 4, p, 4, p, 4, 4, 4, 4, 0, 1, None, None) == ARG
    assert na(p, 8192, p, 8192, p, 8192, 8192, 8192, 8192, 4, 1, None, None) == WS
    # FP64 host pipeline: slice count, slice budget
    hp = lib.ozk_matmul_host_f64
    assert hp(p, 4, p, 4, p, 4, 4, 4, 4, -1, 0, None, 0, None, None) == ARG
    assert hp(p, 4, p, 4, p, 4, 4, 4, 4, -1, 99, None, 0, None, None) == ARG
    assert hp(p, 10000, p, 2, p, 2, 2, 10000, 2, -1, 8, None, 0, None, None) == UNSAFE
    # gram and residual
    gm = lib.ozk_gram_f64
    assert gm(None, 4, p, 4, 4, 4, -1, 4, 1, None, 0, None, None) == ARG
    assert gm(p, 4, p, 4, 0, 4, -1, 4, 1, None, 0, None, None) == ARG
    assert gm(p, 4, p, 3, 4, 4, -1, 4, 1, None, 0, None, None) == ARG
    assert gm(p, 4, p, 4, 4, 0, -1, 4, 1, None, 0, None, None) == OK
    rs = lib.ozk_residual_f64
    assert rs(p, 4, None, 2, p, 2, p, 2, 4, 4, 2, -1, 4, 1, None, 0, None, None) == ARG
    assert rs(p, 4, p, 1, p, 2, p, 2, 4, 4, 2, -1, 4, 1, None, 0, None, None) == ARG
    assert rs(p, 4, p, 2, p, 2, p, 2, 0, 4, 2, -1, 4, 1, None, 0, None, None) == OK
    # accumulation and schedules
    assert lib.ozk_accumulate_2sum(None, p, p, 4, 4, 4, 1, None, None, p, 4, None) == ARG
    assert lib.ozk_accumulate_2sum(p, p, p, 4, 4, 0, 1, None, None, p, 4, None) == ARG
    pa = (ctypes.c_uint8 * 4)()
    pb = (ctypes.c_uint8 * 4)()
    assert lib.ozk_triangular_schedule(0, pa, pb, 4) == ARG
    assert lib.ozk_triangular_schedule(8, pa, pb, 4) == ARG  # 36 pairs do not fit in 4
    # the multi-GPU context and operators: a NULL context or bad arguments are
    # refused before NCCL or CUDA is touched
    vp1 = (ctypes.c_void_p * 1)(p)
    i1 = (ctypes.c_int64 * 1)(4)
    assert lib.ozk_nccl_unique_id(None, 0) == ARG
    assert lib.ozk_context_create_rank(None, 2, 0, p, _lib.OZK_NCCL_ID_BYTES, 0) == ARG
    out = ctypes.c_void_p()
    assert lib.ozk_context_create_rank(ctypes.byref(out), 2, 2, p, _lib.OZK_NCCL_ID_BYTES,
                                       0) == ARG
    assert lib.ozk_context_create_local(ctypes.byref(out), 0, None) == ARG
    assert lib.ozk_context_info(None, None, None, None) == ARG
    assert lib.ozk_context_wait(None, None) == ARG
    assert lib.ozk_context_destroy(None) == OK
    assert lib.ozk_matmul_f64_multi(None, vp1, i1, vp1, i1, vp1, i1, 4, 4, 4, 4, 1,
                                    _lib.OZK_B_REPLICATED, 0, None, None) == ARG
    assert lib.ozk_gram_f64_multi(None, vp1, i1, vp1, i1, 4, 4, 4, 1, 0, None, None) == ARG
    # every refusal leaves a readable detail and a name for its code
    assert _lib.detail()
    for code in (ARG, UNSAFE, WS):
        assert lib.ozk_strerror(code)


def test_log2_table_matches_numpy_log2():
    """The device's exponent rule floor(RN32(log2 m)) (a per-binade threshold
    table) agrees with NumPy's float32 log2 -- the reference's rule,
    ozaki_jax/extract.py:130 -- around every binade edge and at random."""
    txt = open(os.path.join(ROOT, "ozaki_jax_b200", "csrc", "ozk_log2_table.h")).read()
    tab = np.array([int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", txt)], dtype=np.int64)
    assert len(tab) == 277

    def rule(m):
        b = m.view(np.uint32).astype(np.int64)
        sub = -149 + np.floor(np.log2(np.maximum(b, 1).astype(np.float64))).astype(np.int64)
        e = np.where(b >= 0x00800000, (b >> 23) - 127, sub)
        return e + (b >= tab[e + 149])

    ids = []
    for e in range(-149, 128):
        base = int(np.float32(2.0 ** e).view(np.uint32))
        ids.append(np.arange(base - 200, base + 200, dtype=np.int64))
    ids = np.concatenate(ids + [np.random.default_rng(1).integers(1, 0x7F800000, 2_000_000)])
    ids = ids[(ids > 0) & (ids < 0x7F800000)]
    m = ids.astype(np.uint32).view(np.float32)
    ref = np.floor(np.log2(m).astype(np.float32)).astype(np.int64)
    assert np.array_equal(rule(m), ref)
