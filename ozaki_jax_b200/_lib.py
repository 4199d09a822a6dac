"""ctypes binding of libozaki_b200.so (include/ozaki_b200.h).

Loading fails loudly: there is no CPU fallback anywhere in this package.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libozaki_b200.so")

OZK_OK = 0
OZK_ERR_ARG = -1
OZK_ERR_UNSAFE = -2
OZK_ERR_NONFINITE = -3
OZK_ERR_CUDA = -4
OZK_ERR_NCCL = -5
OZK_ERR_TIMEOUT = -6
OZK_ERR_WORKSPACE = -7
OZK_ERR_UNSUPPORTED = -8

OZK_FLAG_NONFINITE = 0x1
OZK_FLAG_TIMEOUT = 0x2
OZK_FLAG_RANGE = 0x4
OZK_FLAG_REDO = 0x8

OZK_B_REPLICATED = 0
OZK_B_ROOT = 1
OZK_B_COLUMNS = 2
OZK_MULTI_NOWAIT = 0x1
OZK_MULTI_BF16 = 0x2
OZK_NCCL_ID_BYTES = 128

OZK_ACC_F64 = 0
OZK_ACC_PRODUCTS = 1
OZK_ACC_FIXED = 2

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_dbl = ctypes.c_double
c_size = ctypes.c_size_t
vp = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/ozaki_b200.h
SIGNATURES = {
    "ozk_compute_rho_f32": (c_int, [c_i64]),
    "ozk_compute_rho_f64": (c_int, [c_i64]),
    "ozk_pair_schedule": (c_int, [c_int, c_int, vp, vp, c_int]),
    "ozk_pair_schedule_snake": (c_int, [c_int, c_int, vp, vp, c_int]),
    "ozk_triangular_schedule": (c_int, [c_int, vp, vp, c_int]),
    "ozk_extract_rows_f64": (c_int, [vp, c_i64, c_i64, c_i64, c_int, c_int, c_int, vp, c_i64, vp,
                                     vp, vp]),
    "ozk_extract_cols_f64": (c_int, [vp, c_i64, c_i64, c_i64, c_int, c_int, c_int, vp, c_i64, vp,
                                     vp, c_size, vp, vp]),
    "ozk_extract_rows_host_f64": (c_int, [vp, c_i64, c_i64, c_i64, c_int, c_int, vp, c_i64, vp,
                                          vp, vp]),
    "ozk_extract_cols_host_f64": (c_int, [vp, c_i64, c_i64, c_i64, c_int, c_int, vp, c_i64, vp,
                                          vp, vp]),
    "ozk_slice_gemm": (c_int, [vp, vp, c_int, vp, vp, c_int, c_i64, c_i64, c_i64, vp, vp, c_int,
                               c_int, c_int, c_dbl, c_dbl, vp, c_i64, vp, c_i64, vp, vp, c_size,
                               c_int, vp, vp]),
    "ozk_slice_gemm_workspace_bytes": (c_size, []),
    "ozk_extract_rows_s8_f64": (c_int, [vp, c_i64, c_i64, c_i64, c_int, c_int, c_int, vp, c_i64,
                                        vp, vp, vp, vp]),
    "ozk_extract_cols_s8_f64": (c_int, [vp, c_i64, c_i64, c_i64, c_int, c_int, c_int, vp, c_i64,
                                        vp, vp, c_size, vp, vp, vp]),
    "ozk_slice_gemm_s8": (c_int, [vp, vp, c_int, vp, vp, c_int, c_i64, c_i64, c_i64, vp, vp, c_int,
                                  c_int, c_dbl, c_dbl, vp, c_i64, vp, c_i64, vp, c_size, c_int, vp,
                                  vp, vp]),
    "ozk_accumulate_2sum": (c_int, [vp, vp, vp, c_i64, c_i64, c_int, c_int, vp, vp, vp, c_i64,
                                    vp]),
    "ozk_accumulate_2sum_scaled": (c_int, [vp, vp, vp, vp, c_int, vp, c_int, c_i64, c_i64, vp, vp,
                                           vp]),
    "ozk_matmul_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_int, c_int]),
    "ozk_matmul_f64": (c_int, [vp, c_i64, vp, c_i64, vp, c_i64, c_i64, c_i64, c_i64, c_int, c_int,
                               c_int, c_int, vp, c_size, vp, vp]),
    "ozk_matmul_hostbuf_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_int, c_int, c_int,
                                                    c_i64]),
    "ozk_matmul_f64_hostbuf": (c_int, [vp, c_i64, vp, c_i64, vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                       c_int, c_int, c_int, c_i64, vp, c_size, vp, vp]),
    "ozk_set_l2_persisting": (c_int, [c_size, vp]),
    "ozk_memcpy_staged": (c_int, [vp, vp, c_size, vp]),
    "ozk_nccl_unique_id": (c_int, [vp, c_size]),
    "ozk_context_create_rank": (c_int, [vp, c_int, c_int, vp, c_size, c_int]),
    "ozk_context_create_local": (c_int, [vp, c_int, vp]),
    "ozk_context_destroy": (c_int, [vp]),
    "ozk_context_info": (c_int, [vp, vp, vp, vp]),
    "ozk_context_wait": (c_int, [vp, vp]),
    "ozk_matmul_f64_multi": (c_int, [vp, vp, vp, vp, vp, vp, vp, c_i64, c_i64, c_i64, c_int,
                                     c_int, c_int, c_int, vp, vp]),
    "ozk_gram_f64_multi": (c_int, [vp, vp, vp, vp, vp, c_i64, c_i64, c_int, c_int, c_int, vp,
                                   vp]),
    "ozk_matmul_f64_noalloc": (c_int, [vp, c_i64, vp, c_i64, vp, c_i64, c_i64, c_i64, c_i64,
                                       c_int, c_int, vp, vp]),
    "ozk_matmul_host_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_int]),
    "ozk_matmul_host_f64": (c_int, [vp, c_i64, vp, c_i64, vp, c_i64, c_i64, c_i64, c_i64, c_int,
                                    c_int, vp, c_size, vp, vp]),
    "ozk_gram_workspace_bytes": (c_size, [c_i64, c_i64, c_int, c_int]),
    "ozk_gram_f64": (c_int, [vp, c_i64, vp, c_i64, c_i64, c_i64, c_int, c_int, c_int, vp, c_size,
                             vp, vp]),
    "ozk_residual_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_int, c_int]),
    "ozk_residual_f64": (c_int, [vp, c_i64, vp, c_i64, vp, c_i64, vp, c_i64, c_i64, c_i64, c_i64,
                                 c_int, c_int, c_int, vp, c_size, vp, vp]),
    "ozk_check_status": (c_int, [vp, vp]),
    "ozk_gemm_stats": (c_int, [vp]),
    "ozk_selftest_timeout": (c_int, [c_int, vp, vp, vp]),
    "ozk_strerror": (ctypes.c_char_p, [c_int]),
    "ozk_last_error_detail": (c_int, [ctypes.c_char_p, c_size]),
    "ozk_version": (ctypes.c_char_p, []),
}

_lib = None


class OzakiError(RuntimeError):
    """A non-argument failure reported by libozaki_b200 (CUDA, timeout, ...)."""

    def __init__(self, code, detail):
        super().__init__(f"{detail} (status {code})")
        self.code = code


def load():
    """Return the loaded library, building it first if it is missing and nvcc
    is available.  Raises RuntimeError when neither works."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        try:
            from . import build as _build
            _build.build()
        except Exception as e:  # pragma: no cover - depends on the host
            raise RuntimeError(
                f"libozaki_b200.so is missing at {LIB_PATH} and could not be built: {e}") from e
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def detail():
    buf = ctypes.create_string_buffer(512)
    load().ozk_last_error_detail(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc):
    """Map a status code to an exception (ValueError for argument / preflight
    problems, as the reference raises them; OzakiError otherwise)."""
    if rc >= 0:
        return rc
    msg = detail() or load().ozk_strerror(rc).decode()
    if rc in (OZK_ERR_ARG, OZK_ERR_UNSAFE, OZK_ERR_NONFINITE):
        raise ValueError(msg)
    if rc == OZK_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise OzakiError(rc, msg)
