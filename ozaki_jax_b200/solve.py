"""FP64-accurate residual b - A @ x (drop-in for ozaki_jax.residual,
ozaki_jax/solve.py:91-151)."""

import torch

from . import _device as D
from . import _lib as L
from .matmul import _PREFIX, _flags_reasons, _read_status, _resolve_precision, compute_rho_f32


def _validate_residual_inputs(A, x, b):
    """ozaki_jax/solve.py:56-75 (same messages)."""
    if D.ndim(A) != 2:
        raise ValueError(f"A must be 2D, got ndim={D.ndim(A)}.")
    N, K = D.shape(A)
    xs, bs = D.shape(x), D.shape(b)
    if len(xs) == 1:
        if xs[0] != K:
            raise ValueError(f"x length {xs[0]} != A columns {K}.")
        if len(bs) != 1 or bs[0] != N:
            raise ValueError(f"b shape {bs} incompatible with A @ x shape ({N},).")
    elif len(xs) == 2:
        if xs[0] != K:
            raise ValueError(f"x rows {xs[0]} != A columns {K}.")
        if len(bs) != 2 or bs[0] != N or bs[1] != xs[1]:
            raise ValueError(f"b shape {bs} incompatible with A @ x shape ({N}, {xs[1]}).")
    else:
        raise ValueError(f"x must be 1D or 2D, got ndim={len(xs)}.")


def _residual_ozaki_device(Ad, Xd, Bd, n_hi, n_lo, rho=None):
    """R = Bd - ozaki(Ad, Xd) on CUDA tensors; returns (R, status)."""
    lib = L.load()
    N, K = Ad.shape
    M = Xd.shape[1]
    dev = Ad.device
    R = torch.empty((N, M), dtype=torch.float64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.ozk_residual_workspace_bytes(N, K, M, n_hi, n_lo)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    L.check(lib.ozk_residual_f64(
        Ad.data_ptr(), Ad.stride(0), Xd.data_ptr(), Xd.stride(0), Bd.data_ptr(), Bd.stride(0),
        R.data_ptr(), R.stride(0), N, K, M, -1 if rho is None else rho, n_hi, n_lo,
        ws.data_ptr(), ws_bytes, status.data_ptr(), D.stream_handle(dev)))
    return R, status


def residual(A, x, b, precision="high", accumulation="bf16_interleaved", mode="f64"):
    """Compute b - A @ x with FP64 accuracy (same type/shape as b).

    mode='f64': native FP64 on the device.  mode='ozaki': the B200 Ozaki
    kernels with rho from K (ozaki_jax/solve.py:143-145); the subtraction is
    fused into the GEMM epilogue (the FP64 running sum starts at b).
    """
    allowed_modes = {"f64", "ozaki"}
    if mode not in allowed_modes:
        raise ValueError(f"mode={mode!r}; expected one of {sorted(allowed_modes)}.")
    if mode == "ozaki":
        allowed_accum = {"bf16_interleaved", "fused"}
        if accumulation not in allowed_accum:
            raise ValueError(
                f"accumulation={accumulation!r}; expected one of {sorted(allowed_accum)}.")
    is_dev = D.is_device_array(A)
    _validate_residual_inputs(A, x, b)
    dev = D.device_of(A, x, b)
    Ad = D.to_device_f64(A, dev)
    Xd = D.to_device_f64(x, dev)
    Bd = D.to_device_f64(b, dev)
    vec = Xd.dim() == 1
    if vec:
        Xd = Xd[:, None].contiguous()
        Bd = Bd[:, None].contiguous()
    if mode == "f64":
        R = Bd - torch.matmul(Ad, Xd)
    else:
        n_hi, n_lo = _resolve_precision(precision)
        N, K = Ad.shape
        if K == 0:
            raise ValueError("zero-size array to reduction operation maximum which has no identity")
        R, status = _residual_ozaki_device(Ad, Xd, Bd, n_hi, n_lo, compute_rho_f32(K))
        flags = _read_status(status)
        if flags:
            raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
    if vec:
        R = R[:, 0]
    return R if is_dev else D.to_host_f64(R)
