"""NumPy-backed stand-in for the parts of `jax` that ozaki-jax imports.

Test infrastructure only: it exists so that the reference implementation
(Efithor/ozaki-jax, pure Python + JAX) can be imported in a container that
has no JAX, to generate golden vectors with the reference's own code.
Nothing in the product imports it.

Semantics: `jit` is the identity; arrays are NumPy arrays, so every FP32 op
is one IEEE round-to-nearest operation (no contraction), which is the
arithmetic the reference's traced programs express.
"""

from . import numpy  # noqa: F401  (jax.numpy)


class Array:  # nothing is ever an instance: NumPy in -> NumPy out
    pass


class _Config:
    _flags = {"jax_enable_x64": True}

    def update(self, name, value):
        self._flags[name] = value

    def read(self, name):
        return self._flags[name]


config = _Config()


def jit(fun=None, **_kw):
    if fun is None:
        return lambda f: f
    return fun


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape, self.dtype = shape, dtype


def block_until_ready(x):
    return x

