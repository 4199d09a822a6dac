"""`jax.scipy` stand-in (test infrastructure only)."""
