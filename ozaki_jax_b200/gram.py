"""FP64-accurate Gram matrix A^T A (drop-in for ozaki_jax.gram,
ozaki_jax/gram.py:47-99)."""

import torch

from . import _device as D
from . import _lib as L
from .matmul import _PREFIX, _flags_reasons, _read_status, _resolve_precision, compute_rho_f32


def _gram_ozaki_device(Ad, n_hi, n_lo, rho=None):
    """G = ozaki(A^T, A), exactly symmetric (tiles on/above the diagonal are
    computed once and mirrored).  Returns (G, status tensor)."""
    lib = L.load()
    N, K = Ad.shape
    dev = Ad.device
    G = torch.empty((K, K), dtype=torch.float64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.ozk_gram_workspace_bytes(N, K, n_hi, n_lo)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    L.check(lib.ozk_gram_f64(Ad.data_ptr(), Ad.stride(0), G.data_ptr(), G.stride(0), N, K,
                             -1 if rho is None else rho, n_hi, n_lo, ws.data_ptr(), ws_bytes,
                             status.data_ptr(), D.stream_handle(dev)))
    return G, status


def gram(A, precision="high", accumulation="bf16_interleaved", mode="f64"):
    """Compute A^T @ A with FP64 accuracy; the result is symmetric.

    mode='f64': native FP64 product on the device, (G + G^T) / 2.
    mode='ozaki': Ozaki product from the B200 kernels (rho from the row count,
    ozaki_jax/gram.py:92-95); accumulation 'bf16_interleaved' and 'fused'
    both run the exact int64 fixed-point epilogue (each element's pair
    products summed exactly, rounded to FP64 once) on the tiles on or above
    the diagonal, each written mirrored, so G is exactly symmetric.
    """
    allowed_modes = {"f64", "ozaki"}
    if mode not in allowed_modes:
        raise ValueError(f"mode={mode!r}; expected one of {sorted(allowed_modes)}.")
    if mode == "ozaki":
        allowed_accum = {"bf16_interleaved", "fused"}
        if accumulation not in allowed_accum:
            raise ValueError(
                f"accumulation={accumulation!r}; expected one of {sorted(allowed_accum)}.")
    if D.ndim(A) != 2:
        raise ValueError(f"A must be 2D, got ndim={D.ndim(A)}.")
    is_dev = D.is_device_array(A)
    dev = D.device_of(A)
    Ad = D.to_device_f64(A, dev)
    if mode == "f64":
        G = torch.matmul(Ad.T, Ad)
        G = (G + G.T) * 0.5
    else:
        n_hi, n_lo = _resolve_precision(precision)
        N, K = Ad.shape
        if N == 0:
            G = torch.zeros((K, K), dtype=torch.float64, device=dev)
        else:
            G, status = _gram_ozaki_device(Ad, n_hi, n_lo, compute_rho_f32(N))
            flags = _read_status(status)
            if flags:
                # the reference has no preflight here and would return NaNs;
                # non-finite input is reported instead of silently propagated
                raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
    return G if is_dev else D.to_host_f64(G)
