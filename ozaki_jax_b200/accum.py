"""The reference's standalone 2Sum accumulation API (ozaki_jax/pallas_ops.py:372-469)
on the device.

`accumulate_2sum` takes the reference's arguments (products, FP32 column and
row scales, the block/group structure) and returns (C_hi, C_lo) bit for bit
as the reference computes them; the 'jax' and 'pallas' backends of the
reference compute the same words, so every backend name maps to one kernel
(`ozk_accumulate_2sum_scaled`).
"""

import ctypes

import numpy as np
import torch

from . import _device as D
from . import _lib as L

_BACKENDS = ("auto", "jax", "pallas")


def accumulate_2sum(products, col_scales, row_scales, block_group_sizes, N=None, M=None,
                    backend="auto"):
    """Scaled FP32 2Sum accumulation (pallas_ops.py:372-396).

    products: (n_products, N, M) FP32; col_scales: (n_products, M) FP32;
    row_scales: (n_groups, N) FP32; block_group_sizes: tuple of tuples of group
    sizes, one tuple per block.  N, M: accepted for the reference's padding
    contract (unused: no padding here).  Returns (C_hi, C_lo), FP32 (N, M);
    device tensors in -> device tensors out, NumPy in -> NumPy out.
    """
    if backend not in _BACKENDS:
        raise ValueError(f"Unknown backend={backend!r}; expected 'auto', 'jax', or 'pallas'.")
    device_in = D.is_device_array(products)
    dev = D.device_of(products, col_scales, row_scales)

    def f32(x):
        if D.is_device_array(x):
            return x.to(device=dev, dtype=torch.float32).contiguous()
        return torch.as_tensor(np.ascontiguousarray(x, dtype=np.float32)).to(dev)

    P, cs, rs = f32(products), f32(col_scales), f32(row_scales)
    if P.dim() != 3:
        raise ValueError("products must be (n_products, N, M)")
    n_prod, n, m = P.shape
    sizes = [int(g) for block in block_group_sizes for g in block]
    ends = np.cumsum([len(block) for block in block_group_sizes]).astype(np.int32)
    if sum(sizes) != n_prod or cs.shape != (n_prod, m) or rs.shape != (len(sizes), n):
        raise ValueError("products, scales and block_group_sizes do not match")
    gs = (ctypes.c_int32 * max(len(sizes), 1))(*sizes)
    be = (ctypes.c_int32 * max(len(ends), 1))(*ends.tolist())
    C_hi = torch.empty((n, m), dtype=torch.float32, device=dev)
    C_lo = torch.empty((n, m), dtype=torch.float32, device=dev)
    L.check(L.load().ozk_accumulate_2sum_scaled(
        P.data_ptr(), cs.data_ptr(), rs.data_ptr(), gs, len(sizes), be, len(ends), n, m,
        C_hi.data_ptr(), C_lo.data_ptr(), D.stream_handle(dev)))
    if device_in:
        return C_hi, C_lo
    return C_hi.cpu().numpy(), C_lo.cpu().numpy()


def validate_accumulation_2sum(N=128, M=128, K=128):
    """The reference's self-check (pallas_ops.py:399-469) on the device: precision
    'max' slice products of seeded N(0,1) inputs (RandomState(42)), accumulated
    in FP64 (the baseline) and by the FP32 2Sum; returns {"match",
    "max_rel_error", "baseline_error", "N", "M", "K"} with match = 2Sum max
    relative error < 1e-9."""
    from .matmul import _ondevice_device, _PRECISION_PRESETS
    rng = np.random.RandomState(42)
    A = rng.randn(N, K).astype(np.float64)
    B = rng.randn(K, M).astype(np.float64)
    C_exact = A @ B
    n_hi, n_lo = _PRECISION_PRESETS["max"]
    dev = D.device_of()
    Ad, Bd = torch.as_tensor(A).to(dev), torch.as_tensor(B).to(dev)
    base, st = _ondevice_device(Ad, Bd, n_hi, n_lo, "host")       # FP64 accumulation
    twosum, st2 = _ondevice_device(Ad, Bd, n_hi, n_lo, "ondevice")  # reference-order 2Sum
    scale = np.max(np.abs(C_exact))
    baseline_err = float(np.max(np.abs(base.cpu().numpy() - C_exact)) / scale)
    twosum_err = float(np.max(np.abs(twosum.cpu().numpy() - C_exact)) / scale)
    return {"match": twosum_err < 1e-9, "max_rel_error": twosum_err,
            "baseline_error": baseline_err, "N": N, "M": M, "K": K}
