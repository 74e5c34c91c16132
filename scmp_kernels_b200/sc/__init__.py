"""Stochastic-computing matmul on B200 (API of scmp_kernels/sc/__init__.py).

* ``sc_matmul`` -- granularity dispatcher (per_tensor / per_row / per_head).
* ``clear_rng_cache`` -- drop cached RNG sequences and device tables (call it
  after changing the SC_OWEN_MODE / SC_DISABLE_OWEN / SC_SCRAMBLE_RESCALE
  environment variables or rotating seeds).
* ``det_kernel_tuning`` -- accepted for compatibility; results do not depend
  on it.
* ``sc_matmul_levels`` -- per-row stream lengths (the caller's mixed-precision
  row levels) in one call.
"""
from .kernels import clear_rng_cache, det_kernel_tuning
from .matmul import sc_matmul
from .levels import sc_matmul_levels
from .prepared import PreparedWeight, prepare_weight, sc_matmul_prepared

__all__ = ["sc_matmul", "clear_rng_cache", "det_kernel_tuning", "PreparedWeight", "prepare_weight",
           "sc_matmul_prepared", "sc_matmul_levels"]
