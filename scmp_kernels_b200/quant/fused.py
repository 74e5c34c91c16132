"""One-launch FP32 -> SC-domain quantisers (API of scmp_kernels/quant/fused.py).

Outputs keep the reference's formats:
  bipolar  -> (boundary int16, sign int8, scale)
  unipolar -> (boundary int32, scale, zp, row_sum or None)
``boundary`` is the quantised magnitude remapped onto the enable grid,
``rint(|x_int| * fl32(rng_levels / q_max))``. Each function is one launch of
a native sm_100a kernel.
"""
from __future__ import annotations

import ctypes
import functools
from typing import Optional

import torch

from .. import _lib


def _resolve_rng_levels(sc_prec: int, rng_levels: Optional[int]) -> int:
    return 2 ** sc_prec if rng_levels is None else int(rng_levels)


def _dev(x: torch.Tensor) -> torch.Tensor:
    if x.device.type != "cuda":
        _lib.require_cuda()
        x = x.cuda()
    return x.float().contiguous()


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(_lib.stream_handle(t.device))


@functools.lru_cache(maxsize=8)
def _quant_dummy(device: torch.device) -> torch.Tensor:
    """1-element placeholder for unused output pointers (fused.py:126-131)."""
    return torch.empty(1, dtype=torch.int8, device=device)


def fused_quantize_bipolar_perrow(fp_tensor: torch.Tensor, sc_prec: int,
                                  rng_levels: Optional[int] = None):
    """Per-row bipolar quant with on-device scales (fused.py:134-159).
    Returns (boundary int16, sign int8, scale_row float32)."""
    x = _dev(fp_tensor)
    rows, cols = x.shape
    G = _resolve_rng_levels(sc_prec, rng_levels)
    boundary = torch.empty(rows, cols, dtype=torch.int16, device=x.device)
    sign = torch.empty(rows, cols, dtype=torch.int8, device=x.device)
    scale_row = torch.empty(rows, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().scmp_fused_quantize_bipolar_perrow(
            x.data_ptr(), rows, cols, sc_prec, G, boundary.data_ptr(), sign.data_ptr(),
            scale_row.data_ptr(), _stream(x)), "fused_quantize_bipolar_perrow")
    return boundary, sign, scale_row


def fused_quantize_bipolar(fp_tensor: torch.Tensor, abs_max: float, sc_prec: int,
                           rng_levels: Optional[int] = None):
    """Per-tensor bipolar quant with a host range (fused.py:162-189).
    Returns (boundary int16, sign int8, scale float)."""
    x = _dev(fp_tensor)
    rows, cols = x.shape
    G = _resolve_rng_levels(sc_prec, rng_levels)
    boundary = torch.empty(rows, cols, dtype=torch.int16, device=x.device)
    sign = torch.empty(rows, cols, dtype=torch.int8, device=x.device)
    scale = ctypes.c_double(0.0)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().scmp_fused_quantize_bipolar(
            x.data_ptr(), rows, cols, float(abs_max), sc_prec, G, boundary.data_ptr(),
            sign.data_ptr(), ctypes.byref(scale), _stream(x)), "fused_quantize_bipolar")
    return boundary, sign, scale.value


def fused_quantize_unipolar(fp_tensor: torch.Tensor, fp_max: float, fp_min: float, sc_prec: int,
                            compute_sum: bool = False, rng_levels: Optional[int] = None):
    """Unipolar quant with a host range (fused.py:192-234).
    Returns (boundary int32, scale, zp, row_sum float32 or None)."""
    x = _dev(fp_tensor)
    rows, cols = x.shape
    G = _resolve_rng_levels(sc_prec, rng_levels)
    boundary = torch.empty(rows, cols, dtype=torch.int32, device=x.device)
    row_sum = torch.empty(rows, dtype=torch.float32, device=x.device) if compute_sum else None
    scale, zp = ctypes.c_double(0.0), ctypes.c_double(0.0)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().scmp_fused_quantize_unipolar(
            x.data_ptr(), rows, cols, float(fp_max), float(fp_min), sc_prec, G,
            boundary.data_ptr(), row_sum.data_ptr() if compute_sum else None,
            ctypes.byref(scale), ctypes.byref(zp), _stream(x)), "fused_quantize_unipolar")
    return boundary, scale.value, float(zp.value), row_sum


def fused_quant_bipolar_batched(fp_tensor: torch.Tensor, inv_scale: torch.Tensor, sc_prec: int,
                                rng_levels: Optional[int] = None):
    """Per-head bipolar quant with a fused transpose: (BH, rows, cols) float32
    -> boundary int16 and sign int8 in (BH, cols, rows) layout, clamped to
    [-2**(p-1), q_max] (fused_quant_bipolar_batched_kernel, fused.py:237-283)."""
    x = _dev(fp_tensor)
    BH, rows, cols = x.shape
    inv = _dev(inv_scale)
    G = _resolve_rng_levels(sc_prec, rng_levels)
    boundary = torch.empty(BH, cols, rows, dtype=torch.int16, device=x.device)
    sign = torch.empty(BH, cols, rows, dtype=torch.int8, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().scmp_fused_quant_bipolar_batched(
            x.data_ptr(), BH, rows, cols, inv.data_ptr(), sc_prec, G, boundary.data_ptr(),
            sign.data_ptr(), _stream(x)), "fused_quant_bipolar_batched")
    return boundary, sign


def _triton_only(name):
    def f(*_a, **_k):
        raise NotImplementedError(
            f"{name} is a Triton kernel object in the reference; scmp_kernels_b200 has no Triton. "
            "Use the function API (fused_quantize_*, fused_quant_bipolar_batched).")
    return f


fused_quant_kernel = _triton_only("fused_quant_kernel")
fused_quant_bipolar_batched_kernel = _triton_only("fused_quant_bipolar_batched_kernel")

__all__ = ["fused_quant_kernel", "fused_quant_bipolar_batched_kernel", "fused_quantize_bipolar",
           "fused_quantize_bipolar_perrow", "fused_quantize_unipolar", "fused_quant_bipolar_batched",
           "_quant_dummy"]
