"""SmoothQuant transform (API of scmp_kernels/quant/smoothquant.py).

``Y = A @ B.T = (A / s) @ (B * s).T`` with per-channel ``s > 0`` moves
activation outliers into the weight. ``sc_matmul(..., smooth_scales=s)``
applies the two diagonal scalings inside its device quantiser; the helpers
below are the calibration side (plain torch, off the hot path) and the
stand-alone transform.
"""
from __future__ import annotations

from typing import Optional

import torch


@torch.no_grad()
def accumulate_act_scales(x: torch.Tensor, running: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Running per-channel max-abs over ``x``'s last axis (smoothquant.py:32-50)."""
    cur = x.detach().abs().reshape(-1, x.shape[-1]).amax(dim=0)
    if running is None:
        return cur.clone()
    return torch.maximum(running.to(device=cur.device, dtype=cur.dtype), cur)


@torch.no_grad()
def compute_smooth_scales(act_scales: torch.Tensor, weight: torch.Tensor, alpha: float = 0.5,
                          eps: float = 1e-5) -> torch.Tensor:
    """``s_j = act_max_j**alpha / w_max_j**(1-alpha)`` clamped at eps (smoothquant.py:53-93)."""
    if not 0.0 <= alpha <= 1.0:
        raise ValueError(f"alpha must be in [0, 1], got {alpha}")
    if act_scales.dim() != 1:
        raise ValueError(f"act_scales must be 1D (D,), got shape {tuple(act_scales.shape)}")
    if weight.dim() != 2:
        raise ValueError(f"weight must be 2D (M, D), got shape {tuple(weight.shape)}")
    if weight.shape[-1] != act_scales.shape[0]:
        raise ValueError(
            f"D mismatch: weight.shape[-1]={weight.shape[-1]} vs act_scales.shape[0]={act_scales.shape[0]}")
    a = act_scales.to(device=weight.device, dtype=weight.dtype).clamp(min=eps)
    w_max = weight.abs().amax(dim=0).clamp(min=eps)
    return (a.pow(alpha) / w_max.pow(1.0 - alpha)).clamp(min=eps)


def _check_smoothing(a: torch.Tensor, b: torch.Tensor, smooth_scales: torch.Tensor) -> None:
    if smooth_scales.dim() != 1:
        raise ValueError(f"smooth_scales must be 1D (D,), got shape {tuple(smooth_scales.shape)}")
    if a.shape[-1] != smooth_scales.shape[0] or b.shape[-1] != smooth_scales.shape[0]:
        raise ValueError(
            f"D mismatch: a.shape[-1]={a.shape[-1]}, b.shape[-1]={b.shape[-1]}, "
            f"smooth_scales.shape[0]={smooth_scales.shape[0]}")


@torch.no_grad()
def apply_smoothing(a: torch.Tensor, b: torch.Tensor, smooth_scales: torch.Tensor):
    """``(a / s, b * s)`` along the last axis (smoothquant.py:96-126)."""
    _check_smoothing(a, b, smooth_scales)
    return (a / smooth_scales.to(device=a.device, dtype=a.dtype),
            b * smooth_scales.to(device=b.device, dtype=b.dtype))


@torch.no_grad()
def apply_smoothing_offline(weight: torch.Tensor, smooth_scales: torch.Tensor) -> torch.Tensor:
    """Bake ``s`` into a weight once: ``weight * s`` (smoothquant.py:129-147)."""
    if smooth_scales.dim() != 1:
        raise ValueError(f"smooth_scales must be 1D (D,), got shape {tuple(smooth_scales.shape)}")
    if weight.shape[-1] != smooth_scales.shape[0]:
        raise ValueError(
            f"D mismatch: weight.shape[-1]={weight.shape[-1]} vs smooth_scales.shape[0]={smooth_scales.shape[0]}")
    return weight * smooth_scales.to(device=weight.device, dtype=weight.dtype)


__all__ = ["accumulate_act_scales", "compute_smooth_scales", "apply_smoothing",
           "apply_smoothing_offline"]
