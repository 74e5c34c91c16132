"""FP32 -> SC-domain quantisation (API of scmp_kernels/quant/__init__.py).

* :mod:`.fused`   -- one-launch per-tensor / per-row / per-head quantisers.
* :mod:`.grouped` -- row-group quantisers of the per_row path.
* :mod:`.smoothquant` -- SmoothQuant calibration helpers and transform.
"""
from .fused import (
    fused_quant_kernel,
    fused_quant_bipolar_batched_kernel,
    fused_quantize_bipolar,
    fused_quantize_bipolar_perrow,
    fused_quantize_unipolar,
    fused_quant_bipolar_batched,
    _quant_dummy,
)
from .grouped import (
    _grouped_symmetric_quant,
    _grouped_asymmetric_quant,
    _grouped_symmetric_quant_batched,
)
from .smoothquant import (
    accumulate_act_scales,
    compute_smooth_scales,
    apply_smoothing,
    apply_smoothing_offline,
)

__all__ = [
    "fused_quant_kernel", "fused_quant_bipolar_batched_kernel", "fused_quantize_bipolar",
    "fused_quantize_bipolar_perrow", "fused_quantize_unipolar", "fused_quant_bipolar_batched",
    "_quant_dummy", "_grouped_symmetric_quant", "_grouped_asymmetric_quant",
    "_grouped_symmetric_quant_batched", "accumulate_act_scales", "compute_smooth_scales",
    "apply_smoothing", "apply_smoothing_offline",
]
