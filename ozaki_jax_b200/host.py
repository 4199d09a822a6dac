"""matmul(pipeline='host'): the reference's FP64 extraction pipeline
(ozaki_jax/matmul.py:77-116, :823-851; ozaki_jax/extract.py:12-103), run on
the device: FP64 sigma-trick slices (n_slices per operand), triangular pair
schedule i + j <= n_slices - 1, FP64 accumulation in the GEMM epilogue."""

import torch

from . import _device as D
from . import _lib as L
from .matmul import _PREFIX, _all_finite, _bound_reasons, _fallback, _flags_reasons
from .matmul import _read_status, _validate_safe_mode, _validate_shapes, compute_rho_f64


def host_safety_reasons(K, n_slices):
    """_ozaki_safety_report without the finiteness scan (matmul.py:77-116)."""
    rho = compute_rho_f64(K)
    bits = 53 - rho
    reasons = _bound_reasons(K, bits, "this BF16->FP32 exactness model")
    if n_slices * max(bits, 0) < 53:
        reasons.append(
            f"insufficient slice budget: n_slices*bits_per_slice={n_slices * max(bits, 0)} < 53")
    return rho, reasons


def matmul_host(A, B, n_slices, safe_mode):
    if n_slices < 1:
        raise ValueError("n_slices must be >= 1.")
    _validate_shapes(A, B)
    N, K = D.shape(A)
    M = D.shape(B)[1]
    rho, reasons = host_safety_reasons(K, n_slices)
    _validate_safe_mode(safe_mode)
    dev = D.device_of(A, B)
    Ad = D.to_device_f64(A, dev)
    Bd = D.to_device_f64(B, dev)
    if reasons:
        if not _all_finite(Ad, Bd):
            reasons.append("inputs contain NaN or Inf")
        if safe_mode == "fallback":
            return _fallback(Ad, Bd)
        raise ValueError(_PREFIX + "; ".join(reasons))
    if N == 0 or M == 0:
        return torch.zeros((N, M), dtype=torch.float64, device=dev)
    if K == 0:
        raise ValueError("zero-size array to reduction operation maximum which has no identity")
    lib = L.load()
    C = torch.empty((N, M), dtype=torch.float64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = lib.ozk_matmul_host_workspace_bytes(N, K, M, n_slices)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    L.check(lib.ozk_matmul_host_f64(
        Ad.data_ptr(), Ad.stride(0), Bd.data_ptr(), Bd.stride(0), C.data_ptr(), C.stride(0),
        N, K, M, rho, n_slices, ws.data_ptr(), ws_bytes, status.data_ptr(),
        D.stream_handle(dev)))
    flags = _read_status(status)
    if flags & L.OZK_FLAG_NONFINITE:
        if safe_mode == "fallback":
            return _fallback(Ad, Bd)
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags & L.OZK_FLAG_NONFINITE)))
    return C
