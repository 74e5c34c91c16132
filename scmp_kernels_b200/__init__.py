"""B200-native (sm_100a) stochastic-computing matmul.

Drop-in for the ``sc_matmul`` path of scmp_kernels: the same Python API
(:func:`sc_matmul`, :func:`clear_rng_cache`, the ``quant`` package) over a
C-ABI library of hand-written CUDA kernels (``libscmp_b200.so``).
"""
from .sc import clear_rng_cache, det_kernel_tuning, prepare_weight, sc_matmul, sc_matmul_levels, sc_matmul_prepared

__all__ = ["sc_matmul", "clear_rng_cache", "det_kernel_tuning", "prepare_weight", "sc_matmul_prepared",
           "sc_matmul_levels"]
