"""FP64-accurate matrix multiplication via the Ozaki scheme on B200.

Drop-in for `ozaki_jax.matmul` (ozaki_jax/matmul.py:781-851): the same
arguments, presets, preflight and error texts.  The on-device pipeline runs
as sm_100a kernels of libozaki_b200.so:

  extract (K1)   FP64 -> double-FP32 split -> BF16 sigma-trick slices, per row
                 of A and per column of B, bit-identical to the reference;
  slice GEMM (K2) persistent tcgen05/TMEM kernel over the pair schedule with
                 the scaled accumulation fused into its epilogue.

Accumulation of the exact per-pair products (the `accumulation` argument):
  'fused', 'bf16_interleaved'  exact int64 fixed-point sums per element (unit
                               2^-36 of the top slices' product grid), rounded
                               to FP64 once -- no FP64 work per pair, which
                               keeps the tensor cores fed; its resolution
                               (about 2^-50 * max|A[r,:]| * max|B[:,c]|) is far
                               below the Ozaki truncation error of every preset;
  'host'                       FP64 sums in pair order: the semantics of the
                               reference's FP64 host accumulation;
  'ondevice'                   materialised products + the reference's FP32 2Sum
                               in the reference's order: the reference's fused /
                               ondevice result bit for bit.
"""

import ctypes

import numpy as np
import torch

from . import _device as D
from . import _lib as L

# On-device pipeline precision presets (ozaki_jax/matmul.py:168-172).
_PRECISION_PRESETS = {
    "high": (4, 1),    # 24 GEMMs
    "medium": (3, 1),  # 15 GEMMs
    "max": (5, 4),     # 65 GEMMs
}

_ACCUMULATIONS = {"fused", "bf16_interleaved", "ondevice", "host"}
_SAFE_MODES = {"raise", "fallback"}
_PREFIX = "Ozaki preflight marked this input as unsafe: "


def _resolve_precision(precision):
    """Preset name or custom (n_hi, n_lo) tuple (ozaki_jax/matmul.py:175-194)."""
    if isinstance(precision, tuple) and len(precision) == 2:
        n_hi, n_lo = precision
        if n_hi < 1 or n_lo < 1:
            raise ValueError(
                f"Custom precision tuple must have n_hi >= 1 and n_lo >= 1, "
                f"got ({n_hi}, {n_lo})."
            )
        return precision
    if precision not in _PRECISION_PRESETS:
        raise ValueError(
            f"Unknown precision={precision!r}; expected one of "
            f"{sorted(_PRECISION_PRESETS)} or a (n_hi, n_lo) tuple."
        )
    return _PRECISION_PRESETS[precision]


def _validate_accumulation_mode(accumulation):
    if accumulation not in _ACCUMULATIONS:
        raise ValueError(
            f"Unknown accumulation={accumulation!r}; expected one of {sorted(_ACCUMULATIONS)}."
        )


def _validate_safe_mode(safe_mode):
    if safe_mode not in _SAFE_MODES:
        raise ValueError(
            f"Invalid safe_mode={safe_mode!r}; expected one of {sorted(_SAFE_MODES)}."
        )


def _validate_shapes(A, B):
    """ozaki_jax/matmul.py:67-74."""
    if D.ndim(A) != 2 or D.ndim(B) != 2:
        raise ValueError("Inputs must be rank-2 matrices.")
    if D.shape(A)[1] != D.shape(B)[0]:
        raise ValueError(
            f"Incompatible shapes for matmul: {D.shape(A)} and {D.shape(B)}."
        )


def compute_rho_f32(K):
    """_compute_rho_f32 (ozaki_jax/extract.py:109-113), evaluated by the library."""
    return int(L.load().ozk_compute_rho_f32(int(K)))


def compute_rho_f64(K):
    """_compute_rho (ozaki_jax/extract.py:12-18)."""
    return int(L.load().ozk_compute_rho_f64(int(K)))


def _bound_reasons(K, bits, what):
    """The K / bits part of the preflight (ozaki_jax/matmul.py:605-621, :84-97)."""
    reasons = []
    if bits <= 0:
        reasons.append(
            f"non-positive bits per slice ({bits}); K={K} is too large for {what}")
    elif K * (2 ** bits - 1) ** 2 >= 2 ** 24:
        max_K = int(2 ** 24 / (2 ** bits - 1) ** 2)
        reasons.append(
            f"K={K} violates BF16->FP32 exact inner-product bound (need K <= {max_K})")
    return reasons


def ondevice_safety_report(A, B, n_hi=4, n_lo=1):
    """_ondevice_safety_report (ozaki_jax/matmul.py:600-638).  The finiteness
    scan runs on the device (one reduction) instead of on the host."""
    _validate_shapes(A, B)
    K = D.shape(A)[1]
    rho = compute_rho_f32(K)
    bits = 24 - rho
    reasons = _bound_reasons(K, bits, "FP32 extraction")
    if not _all_finite(A, B):
        reasons.append("inputs contain NaN or Inf")
    return {"safe": not reasons, "rho": rho, "bits_per_slice": bits, "n_hi": n_hi,
            "n_lo": n_lo, "n_gemms": n_hi * n_hi + n_hi * n_lo + n_lo * n_hi,
            "reasons": reasons}


def _all_finite(*xs):
    ok = True
    for x in xs:
        if D.is_device_array(x):
            ok = ok and bool(torch.isfinite(x).all())
        else:
            ok = ok and bool(np.isfinite(np.asarray(x, dtype=np.float64)).all())
    return ok


def _fallback(Ad, Bd):
    """safe_mode='fallback': plain FP64 A @ B (ozaki_jax/matmul.py:133-134),
    computed on the device."""
    return torch.matmul(Ad, Bd)


def _flags_reasons(flags):
    reasons = []
    if flags & L.OZK_FLAG_NONFINITE:
        reasons.append("inputs contain NaN or Inf")
    if flags & L.OZK_FLAG_RANGE:
        reasons.append("inputs exceed the FP32 range, so the double-FP32 split overflows")
    return reasons


def _read_status(status):
    flags = int(status.item())
    if flags & L.OZK_FLAG_TIMEOUT:
        raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
    return flags


def _ondevice_device(Ad, Bd, n_hi, n_lo, accumulation, rho=None, out=None):
    """Run the on-device pipeline on CUDA float64 tensors; returns (C, flags
    tensor).  Nothing is synchronised here."""
    lib = L.load()
    N, K = Ad.shape
    M = Bd.shape[1]
    dev = Ad.device
    C = out if out is not None else torch.empty((N, M), dtype=torch.float64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    mode = _acc_mode(accumulation)
    ws_bytes = lib.ozk_matmul_workspace_bytes(N, K, M, n_hi, n_lo)
    if mode == L.OZK_ACC_PRODUCTS:
        ws_bytes += (n_hi * n_hi + 2 * n_hi * n_lo) * N * M * 4 + 256
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    L.check(lib.ozk_matmul_f64(
        Ad.data_ptr(), Ad.stride(0), Bd.data_ptr(), Bd.stride(0), C.data_ptr(), C.stride(0),
        N, K, M, -1 if rho is None else rho, n_hi, n_lo, mode, ws.data_ptr(), ws_bytes,
        status.data_ptr(), D.stream_handle(dev)))
    return C, status


def _acc_mode(accumulation):
    return {"ondevice": L.OZK_ACC_PRODUCTS, "host": L.OZK_ACC_F64}.get(accumulation,
                                                                      L.OZK_ACC_FIXED)


def _ondevice_hostbuf(A, B, n_hi, n_lo, accumulation, rho, dev):
    """NumPy in -> NumPy out through ozk_matmul_f64_hostbuf: the library copies
    A and B in and C out itself, overlapping the copies with the compute.
    Returns (C as a NumPy array, OZK_FLAG_* bits)."""
    lib = L.load()
    Ah = np.ascontiguousarray(A, dtype=np.float64)
    Bh = np.ascontiguousarray(B, dtype=np.float64)
    N, K = Ah.shape
    M = Bh.shape[1]
    Ch = D.host_empty_f64((N, M))
    mode = _acc_mode(accumulation)
    with torch.cuda.device(dev):
        ws_bytes = lib.ozk_matmul_hostbuf_workspace_bytes(N, K, M, n_hi, n_lo, mode, 0)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        flags = ctypes.c_int32(0)
        L.check(lib.ozk_matmul_f64_hostbuf(
            Ah.ctypes.data, K, Bh.ctypes.data, M, Ch.ctypes.data, M, N, K, M, rho, n_hi, n_lo,
            mode, 0, ws.data_ptr(), ws_bytes, ctypes.byref(flags), D.stream_handle(dev)))
        del ws
    if flags.value & L.OZK_FLAG_TIMEOUT:
        raise L.OzakiError(L.OZK_ERR_TIMEOUT, "a device-side wait exceeded its time budget")
    return Ch, flags.value


def _matmul_ondevice(A, B, safe_mode, accumulation, n_hi, n_lo):
    """_matmul_ondevice (ozaki_jax/matmul.py:641-728) on the B200 kernels."""
    _validate_accumulation_mode(accumulation)
    _validate_shapes(A, B)
    N, K = D.shape(A)
    M = D.shape(B)[1]
    rho = compute_rho_f32(K)
    bits = 24 - rho
    reasons = _bound_reasons(K, bits, "FP32 extraction")
    _validate_safe_mode(safe_mode)
    dev = D.device_of(A, B)
    if not D.is_device_array(A) and not reasons and N > 0 and M > 0 and K > 0:
        C, flags = _ondevice_hostbuf(A, B, n_hi, n_lo, accumulation, rho, dev)
        if not flags:
            return C
        if safe_mode == "fallback":
            return _fallback(D.to_device_f64(A, dev), D.to_device_f64(B, dev))
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
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
    C, status = _ondevice_device(Ad, Bd, n_hi, n_lo, accumulation, rho)
    flags = _read_status(status)
    if flags:
        if safe_mode == "fallback":
            return _fallback(Ad, Bd)
        raise ValueError(_PREFIX + "; ".join(_flags_reasons(flags)))
    return C


def matmul(A, B, n_slices=8, safe_mode="raise", pipeline="host",
           accumulation="fused", precision="high"):
    """FP64 matmul via Ozaki extraction (drop-in for ozaki_jax.matmul).

    A, B: both NumPy arrays (-> NumPy result) or both CUDA tensors (-> CUDA
    tensor on the same device).
    pipeline: 'ondevice' (BF16 slices, preset precision; the B200 hot path)
        or 'host' (FP64 extraction into n_slices slices, triangular pairs).
    accumulation: 'fused' (default), 'bf16_interleaved', 'ondevice', 'host'.
    precision: 'high' (24 GEMMs), 'medium' (15), 'max' (65) or (n_hi, n_lo).
    safe_mode: 'raise' -> ValueError on unsafe input; 'fallback' -> plain
        FP64 A @ B.
    """
    if not D.same_family(A, B):
        raise ValueError("A and B must both be numpy arrays or both be JAX arrays.")
    input_is_device = D.is_device_array(A)

    if pipeline == "ondevice":
        n_hi, n_lo = _resolve_precision(precision)
        C = _matmul_ondevice(A, B, safe_mode, accumulation, n_hi, n_lo)
    elif pipeline == "host":
        from .host import matmul_host
        C = matmul_host(A, B, n_slices, safe_mode)
    else:
        raise ValueError(f"Unknown pipeline={pipeline!r}; expected 'host' or 'ondevice'.")
    if input_is_device or isinstance(C, np.ndarray):
        return C
    return D.to_host_f64(C)


def matmul_numpy(A_f64, B_f64, n_slices=8, safe_mode="raise", pipeline="host",
                 precision="high"):
    """The reference's NumPy pipeline (matmul_numpy, ozaki_jax/matmul.py:854-895) with
    its semantics, computed on the device; always returns a NumPy array.

    pipeline='ondevice': FP32 double split, BF16 slices, exact products summed in
    FP64 (the reference's _accumulate_block_products) -> accumulation='host'.
    pipeline='host': FP64 slices with triangular pairs (matmul(pipeline='host')).
    """
    A = np.asarray(A_f64, dtype=np.float64)
    B = np.asarray(B_f64, dtype=np.float64)
    if pipeline == "ondevice":
        n_hi, n_lo = _resolve_precision(precision)
        C = _matmul_ondevice(A, B, safe_mode, "host", n_hi, n_lo)
    elif pipeline == "host":
        from .host import matmul_host
        C = matmul_host(A, B, n_slices, safe_mode)
    else:
        raise ValueError(f"Unknown pipeline={pipeline!r}; expected 'host' or 'ondevice'.")
    return C if isinstance(C, np.ndarray) else D.to_host_f64(C)
