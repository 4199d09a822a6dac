"""Slice extraction on the device (the parity-test surface of K1).

Drop-ins for ozaki_jax.f32_extract_split_rows / _cols and
jax_extract_split_rows / _cols (ozaki_jax/extract.py:116-191, :197-286).
An FP32 input splits into hi = x, lo = 0, so extracting n slices of an FP32
matrix is the hi half of the library's double-FP32 extraction.
"""

import numpy as np
import torch

from . import _device as D
from . import _lib as L


def _bf16_to_f32(u16):
    return (u16.to(torch.int32) << 16).view(torch.float32)


def extract_device(X, rho, n_hi, n_lo, axis):
    """Double-FP32 split + sigma-trick extraction of a CUDA float64 matrix.

    axis=1: per row, slices (n_hi+n_lo, rows, K); axis=0: per column, slices
    (n_hi+n_lo, cols, K) -- transposed, K contiguous, as the GEMM reads them.
    Returns (slices as BF16 bit patterns int16 tensor, k_pad, int32 exponents,
    status tensor).  Asynchronous.
    """
    lib = L.load()
    dev = X.device
    if axis == 1:
        lines, K = X.shape
    else:
        K, lines = X.shape
    k_pad = (max(K, 1) + 63) // 64 * 64
    ns = n_hi + n_lo
    slices = torch.empty((ns, lines, k_pad), dtype=torch.int16, device=dev)
    exps = torch.empty((ns, lines), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if axis == 1:
        L.check(lib.ozk_extract_rows_f64(X.data_ptr(), X.stride(0), lines, K, rho, n_hi, n_lo,
                                         slices.data_ptr(), k_pad, exps.data_ptr(),
                                         status.data_ptr(), D.stream_handle(dev)))
    else:
        scratch = torch.empty(lines * K, dtype=torch.float64, device=dev)
        L.check(lib.ozk_extract_cols_f64(X.data_ptr(), X.stride(0), K, lines, rho, n_hi, n_lo,
                                         slices.data_ptr(), k_pad, exps.data_ptr(),
                                         scratch.data_ptr(), scratch.numel() * 8,
                                         status.data_ptr(), D.stream_handle(dev)))
    return slices, k_pad, exps, status


def _extract_f32(X_f32, rho, n_slices, axis):
    if n_slices < 1:
        raise ValueError("n_slices must be >= 1")
    dev = D.device_of(X_f32)
    if D.is_device_array(X_f32):
        Xd = X_f32.to(device=dev, dtype=torch.float32).to(torch.float64).contiguous()
    else:
        Xd = D.to_device_f64(np.asarray(X_f32, dtype=np.float32), dev)
    if Xd.dim() != 2:
        raise ValueError("X must be 2D")
    K = Xd.shape[1] if axis == 1 else Xd.shape[0]
    slices, k_pad, exps, _ = extract_device(Xd, int(rho), int(n_slices), 0, axis)
    S = _bf16_to_f32(slices[:, :, :K])
    if axis == 0:
        S = S.transpose(1, 2)
    return S.contiguous(), exps.to(torch.float32)


def f32_extract_split_rows(X_f32, rho, n_slices=5):
    """Row-scaled slices of an FP32 matrix: (list of FP32 slices, list of FP32
    exponent vectors), NumPy in -> NumPy out."""
    S, E = _extract_f32(X_f32, rho, n_slices, 1)
    if D.is_device_array(X_f32):
        return list(S), list(E)
    S, E = S.cpu().numpy(), E.cpu().numpy()
    return [S[i] for i in range(len(S))], [E[i] for i in range(len(E))]


def f32_extract_split_cols(X_f32, rho, n_slices=5):
    """Column-scaled slices of an FP32 matrix (see f32_extract_split_rows)."""
    S, E = _extract_f32(X_f32, rho, n_slices, 0)
    if D.is_device_array(X_f32):
        return list(S), list(E)
    S, E = S.cpu().numpy(), E.cpu().numpy()
    return [S[i] for i in range(len(S))], [E[i] for i in range(len(E))]


def jax_extract_split_rows(X_f32, rho, n_slices=5):
    """Stacked variant: ((n_slices, N, K) slices, (n_slices, N) exponents) on
    the device."""
    return _extract_f32(X_f32, rho, n_slices, 1)


def jax_extract_split_cols(X_f32, rho, n_slices=5):
    """Stacked variant: ((n_slices, K, M) slices, (n_slices, M) exponents)."""
    return _extract_f32(X_f32, rho, n_slices, 0)


def _extract_f64(X_f64, rho, n_slices, axis):
    """FP64 sigma-trick extraction of the host pipeline on the device:
    (slices (n, lines, K) FP32, exponents (n, lines) FP64)."""
    n_slices = int(n_slices)
    if n_slices < 1:
        raise ValueError("n_slices must be >= 1")
    lib = L.load()
    dev = D.device_of(X_f64)
    Xd = D.to_device_f64(X_f64, dev)
    if Xd.dim() != 2:
        raise ValueError("X must be 2D")
    lines, K = (Xd.shape if axis == 1 else Xd.shape[::-1])
    k_pad = (max(K, 1) + 63) // 64 * 64
    slices = torch.empty((n_slices, lines, k_pad), dtype=torch.int16, device=dev)
    exps = torch.empty((n_slices, lines), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if lines > 0 and K > 0:
        fn = lib.ozk_extract_rows_host_f64 if axis == 1 else lib.ozk_extract_cols_host_f64
        L.check(fn(Xd.data_ptr(), Xd.stride(0), *((lines, K) if axis == 1 else (K, lines)),
                   int(rho), n_slices, slices.data_ptr(), k_pad, exps.data_ptr(),
                   status.data_ptr(), D.stream_handle(dev)))
    S = _bf16_to_f32(slices[:, :, :K])
    if axis == 0:
        S = S.transpose(1, 2)
    return S.contiguous(), exps.to(torch.float64)


def _as_lists(S, E, device_in):
    if device_in:
        return list(S), list(E)
    S, E = S.cpu().numpy(), E.cpu().numpy()
    return [S[i] for i in range(len(S))], [E[i] for i in range(len(E))]


def extract_split_rows(X_f64, rho, n_slices=8):
    """Row-scaled FP64 sigma-trick slices of the host pipeline
    (extract_split_rows, ozaki_jax/extract.py:21-65): (list of FP32 slices
    (N, K), list of FP64 exponent vectors (N,)), NumPy in -> NumPy out."""
    S, E = _extract_f64(X_f64, rho, n_slices, 1)
    return _as_lists(S, E, D.is_device_array(X_f64))


def extract_split_cols(X_f64, rho, n_slices=8):
    """Column-scaled FP64 slices (extract_split_cols, ozaki_jax/extract.py:68-103):
    (list of FP32 slices (K, M), list of FP64 exponent vectors (M,))."""
    S, E = _extract_f64(X_f64, rho, n_slices, 0)
    return _as_lists(S, E, D.is_device_array(X_f64))
