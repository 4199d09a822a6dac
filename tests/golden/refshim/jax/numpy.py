"""`jax.numpy` stand-in: NumPy with JAX's dtype-cast call style.

Test infrastructure only (see the package docstring).
"""

import ml_dtypes as _mld
import numpy as _np
from numpy import *  # noqa: F401,F403
from numpy import linalg  # noqa: F401



class _Cast:
    """A dtype that, like jnp.float32(x), casts arrays without dropping shape
    (NumPy's scalar types turn size-1 arrays into scalars)."""

    def __init__(self, t):
        self._t = t
        self.dtype = _np.dtype(t)

    def __call__(self, x):
        if _np.ndim(x) == 0 and not isinstance(x, _np.ndarray):
            return self._t(x)
        return _np.asarray(x).astype(self._t)


float32 = _Cast(_np.float32)
float64 = _Cast(_np.float64)
int32 = _Cast(_np.int32)
bfloat16 = _Cast(_mld.bfloat16)


def asarray(x, dtype=None):
    return _np.asarray(x, dtype=dtype)


def array(x, dtype=None):
    return _np.array(x, dtype=dtype)


def ldexp(x, n):
    x = _np.asarray(x)
    return _np.ldexp(x, _np.asarray(n).astype(_np.int32)).astype(x.dtype)


def matmul(a, b, preferred_element_type=None):
    a, b = _np.asarray(a), _np.asarray(b)
    if a.dtype == _mld.bfloat16 or b.dtype == _mld.bfloat16:
        a, b = a.astype(_np.float32), b.astype(_np.float32)
    out = _np.matmul(a, b)
    if preferred_element_type is not None:
        out = out.astype(preferred_element_type)
    return out


def dot(a, b, preferred_element_type=None):
    return matmul(a, b, preferred_element_type)
