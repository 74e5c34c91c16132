"""Public ``sc_matmul`` entry point (API of scmp_kernels/sc/matmul.py).

Same signature, defaults, argument gates and error messages as the reference;
dispatch goes to the native B200 path in :mod:`.kernels`.
"""
from __future__ import annotations

import contextlib
import functools
from typing import Optional

import torch

from ..quant.smoothquant import _check_smoothing
from .kernels import (
    _sc_matmul_per_head_bipolar,
    _sc_matmul_per_row,
    _sc_matmul_per_row_batched,
    _sc_matmul_per_row_mlp,
    _sc_matmul_per_tensor,
)

_VALID_GRANULARITIES = ("per_tensor", "per_row", "per_head")
_VALID_MODES = ("bipolar", "unipolar")


def _pin_to_operand_device(fn):
    """Run on the operands' CUDA device and restore the caller's current
    device afterwards (matmul.py:37-58)."""
    @functools.wraps(fn)
    def wrapper(a, b, *args, **kwargs):
        if a.device != b.device:
            raise ValueError(
                f"sc_matmul: a and b must be on the same device, got a.device={a.device}, b.device={b.device}.")
        if a.is_cuda:
            with torch.cuda.device(a.device):
                return fn(a, b, *args, **kwargs)
        return fn(a, b, *args, **kwargs)
    return wrapper


@_pin_to_operand_device
@torch.no_grad()
def sc_matmul(a: torch.Tensor, b: torch.Tensor, *args, **kwargs) -> torch.Tensor:
    """Stochastic-computing matmul ``a @ b.T``; see :func:`_sc_matmul_impl`."""
    guard = torch.cuda.device(a.device) if a.is_cuda else contextlib.nullcontext()
    with guard:
        return _sc_matmul_impl(a, b, *args, **kwargs)


@torch.no_grad()
def _sc_matmul_impl(
    a: torch.Tensor,
    b: torch.Tensor,
    granularity: str = "per_row",
    *,
    mode: str = "bipolar",
    sc_prec: int = 8,
    stoc_len: Optional[int] = None,
    chunk_d: int = 0,
    group_a: int = 1,
    group_b: int = 1,
    rng_levels: Optional[int] = None,
    config: Optional[dict] = None,
    halve_bipolar_stoc_len: bool = False,
    smooth_scales: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Stochastic-computing matmul ``a @ b.T`` (matmul.py:81-279).

    a, b: ``(N, D)`` / ``(M, D)`` or ``(BH, N, D)`` / ``(BH, M, D)``.
    granularity: "per_tensor" | "per_row" | "per_head" quantisation scope.
    mode: "bipolar" (sign-magnitude, q_max = 2**(p-1)-1) or "unipolar"
        (zero point, q_max = 2**p-1).
    sc_prec: p; stoc_len: stream length (default 2**p); rng_levels: enable
        grid (default 2**p); chunk_d > 0: per_row + bipolar + 2D only, per-chunk
        quantisation with float32 accumulation across chunks; group_a/group_b:
        per_row row-group sizes; config: RNG/SNG config (Sobol default);
        halve_bipolar_stoc_len: bipolar stoc_len / rng_levels left at None
        become 2**(p-1); smooth_scales: ``(D,)`` SmoothQuant vector, computes
        ``(a / s) @ (b * s).T``.

    Returns float32 ``(N, M)`` or ``(BH, N, M)`` on the inputs' device.
    Raises ValueError for the same argument combinations as the reference.
    """
    if granularity not in _VALID_GRANULARITIES:
        raise ValueError(
            f"sc_matmul: unknown granularity '{granularity}'. "
            f"Expected one of {_VALID_GRANULARITIES}.")
    if mode not in _VALID_MODES:
        raise ValueError(
            f"sc_matmul: unknown mode '{mode}'. "
            f"Expected one of {_VALID_MODES}.")

    if halve_bipolar_stoc_len and mode == "bipolar":
        halved = 2 ** (sc_prec - 1)
        if stoc_len is None:
            stoc_len = halved
        if rng_levels is None:
            rng_levels = halved

    if smooth_scales is not None:
        _check_smoothing(a, b, smooth_scales)

    if chunk_d > 0:
        if granularity != "per_row":
            raise ValueError(
                f"sc_matmul: chunk_d > 0 requires granularity='per_row', "
                f"got '{granularity}'. D-chunking is only implemented in the "
                f"per-row MLP fast path.")
        if mode != "bipolar":
            raise ValueError(
                f"sc_matmul: chunk_d > 0 requires mode='bipolar', got '{mode}'. "
                f"D-chunking is not implemented for unipolar quantization.")
        if a.dim() != 2 or b.dim() != 2:
            raise ValueError(
                f"sc_matmul: chunk_d > 0 requires 2D inputs (the per-row MLP "
                f"fast path is 2D only), got a.dim()={a.dim()}, b.dim()={b.dim()}.")

    if granularity == "per_head":
        if a.dim() != 3 or b.dim() != 3:
            raise ValueError(
                f"sc_matmul: granularity='per_head' requires 3D inputs (BH, *, D), "
                f"got a.dim()={a.dim()}, b.dim()={b.dim()}.")
        if mode != "bipolar":
            raise ValueError(
                f"sc_matmul: granularity='per_head' currently only supports "
                f"mode='bipolar', got '{mode}'.")

    kw = dict(sc_prec=sc_prec, config=config, stoc_len=stoc_len, rng_levels=rng_levels,
              smooth_scales=smooth_scales)
    if granularity == "per_tensor":
        return _sc_matmul_per_tensor(a, b, mode=mode, **kw)
    if granularity == "per_row":
        if chunk_d > 0:
            return _sc_matmul_per_row_mlp(a, b, mode=mode, group_a=group_a, group_b=group_b,
                                          chunk_d=chunk_d, **kw)
        if a.dim() == 3:
            return _sc_matmul_per_row_batched(a, b, group_a=group_a, group_b=group_b, mode=mode, **kw)
        return _sc_matmul_per_row(a, b, group_a=group_a, group_b=group_b, mode=mode, **kw)
    return _sc_matmul_per_head_bipolar(a, b, **kw)
