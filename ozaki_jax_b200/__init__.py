"""ozaki-jax on B200: FP64-accurate matmul / gram / residual from BF16
tensor-core GEMMs (Ozaki scheme), as sm_100a kernels behind a drop-in
version of ozaki-jax's Python API.

The compute runs in libozaki_b200.so (include/ozaki_b200.h); this package
validates arguments exactly like the reference, moves arrays, and calls it.
There is no CPU fallback: without a CUDA device or the library, calls raise.
"""

__version__ = "0.1.0"

from .matmul import (matmul, matmul_numpy, compute_rho_f32, compute_rho_f64,
                     ondevice_safety_report)
from .gram import gram
from .solve import residual
from .extract import (
    extract_split_rows, extract_split_cols,
    f32_extract_split_rows, f32_extract_split_cols,
    jax_extract_split_rows, jax_extract_split_cols,
)
from .accum import accumulate_2sum, validate_accumulation_2sum

__all__ = [
    "matmul", "matmul_numpy", "gram", "residual",
    "extract_split_rows", "extract_split_cols",
    "f32_extract_split_rows", "f32_extract_split_cols",
    "jax_extract_split_rows", "jax_extract_split_cols",
    "accumulate_2sum", "validate_accumulation_2sum",
    "compute_rho_f32", "compute_rho_f64", "ondevice_safety_report",
]
