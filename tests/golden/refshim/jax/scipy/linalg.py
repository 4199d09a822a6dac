"""`jax.scipy.linalg` stand-in (test infrastructure only)."""
from scipy.linalg import solve_triangular  # noqa: F401
