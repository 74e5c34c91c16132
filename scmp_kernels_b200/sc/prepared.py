"""Static weights: the weight operand b quantised once for repeated per_row calls.

In a served model the second operand of a linear layer (b, the weight) does not
change between calls, yet ``sc_matmul`` quantises it on every call, as the
reference does (``sc/kernels.py:1573-1707``): for a 11008x4096 weight that is a
180 MB read per call, as long as the whole GEMM when a holds a few rows (a
decode step). :func:`prepare_weight` keeps b's quantised operand and row
parameters in a device workspace owned by the returned object, and
:func:`sc_matmul_prepared` runs the per_row path on them (the library's
``SCMP_FLAG_B_READY``). Results are the bits ``sc_matmul(a, b, "per_row", ...)``
gives for the same arguments. This is the static-weight quantisation cache
that the reference's offline SmoothQuant helper
(``quant/smoothquant.py:129-147``) anticipates; the reference has no such API.

A prepared weight refers to b on the device (no copy when b already is a
contiguous float32 CUDA tensor) and owns one workspace. b is quantised on the
first call and again whenever a call needs a larger workspace (more rows of a
than any call before), so b must stay unchanged while the weight is in use;
calls on one weight must be ordered on one stream (two calls in flight at
once on different streams would race on the workspace).
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _lib
from . import kernels as K


class PreparedWeight:
    """b quantised for per_row calls; create with :func:`prepare_weight`."""

    def __init__(self, b, mode, sc_prec, stoc_len, rng_levels, config, group_b, smooth):
        self.b = b                    # float32 (M, D) on the device
        self.mode = mode
        self.sc_prec = sc_prec
        self.group_b = group_b
        self.smooth = smooth          # float32 (D,) on the device, or None
        self.tables = K._get_cached_enable_tables(K._default_config(config, b.shape[1], sc_prec),
                                                  sc_prec, b.device, stoc_len, rng_levels)
        self.workspace: Optional[torch.Tensor] = None
        self.ready = False            # the workspace holds b's quantised operand

    @property
    def shape(self):
        return tuple(self.b.shape)

    @property
    def device(self):
        return self.b.device


@torch.no_grad()
def prepare_weight(b: torch.Tensor, *, mode: str = "bipolar", sc_prec: int = 8,
                   stoc_len: Optional[int] = None, group_b: int = 1, rng_levels: Optional[int] = None,
                   config: Optional[dict] = None, halve_bipolar_stoc_len: bool = False,
                   smooth_scales: Optional[torch.Tensor] = None) -> PreparedWeight:
    """Prepare the weight ``b`` (M, D) of per_row calls ``sc_matmul(a, b, "per_row", ...)``.

    The keyword arguments are those of ``sc_matmul`` that concern b (and the
    RNG configuration); ``group_a`` is given per call. b is copied to the CUDA
    device as float32 (the weight refers to b itself when it already is a
    contiguous float32 CUDA tensor); with ``smooth_scales`` b must be float32 (the
    reference smooths other dtypes in their own precision before the call).
    Quantisation happens on the first :func:`sc_matmul_prepared` call.
    """
    if mode not in ("bipolar", "unipolar"):
        raise ValueError(f"prepare_weight: unknown mode '{mode}'. Expected one of ('bipolar', 'unipolar').")
    if b.dim() != 2:
        raise ValueError(f"prepare_weight: b must be 2D (M, D), got {b.dim()}D")
    if halve_bipolar_stoc_len and mode == "bipolar":
        if stoc_len is None:
            stoc_len = 2 ** (sc_prec - 1)
        if rng_levels is None:
            rng_levels = 2 ** (sc_prec - 1)
    smooth = None
    if smooth_scales is not None:
        if b.dtype != torch.float32:
            raise ValueError("prepare_weight: smooth_scales needs a float32 b")
        if smooth_scales.dim() != 1 or smooth_scales.shape[0] != b.shape[1]:
            raise ValueError(f"prepare_weight: smooth_scales must be ({b.shape[1]},), "
                             f"got {tuple(smooth_scales.shape)}")
    bd = K._to_device(b)
    with torch.cuda.device(bd.device):
        if smooth_scales is not None:
            smooth = K._to_device(smooth_scales.to(device=bd.device, dtype=torch.float32))
        return PreparedWeight(bd, mode, sc_prec, stoc_len, rng_levels, config, group_b, smooth)


@torch.no_grad()
def sc_matmul_prepared(a: torch.Tensor, w: PreparedWeight, *, group_a: int = 1) -> torch.Tensor:
    """``sc_matmul(a, b, "per_row", ...)`` for the prepared weight ``w`` of b.

    a: (N, D), float32 when ``w`` was prepared with smooth_scales. Returns
    float32 (N, M) on a's device (host operands are copied to w's device and
    the result back, as ``sc_matmul`` does).
    """
    if a.dim() != 2:
        raise ValueError(f"sc_matmul_prepared: a must be 2D (N, D), got {a.dim()}D")
    if a.shape[1] != w.b.shape[1]:
        raise ValueError(f"sc_matmul_prepared: inner dimension mismatch: a has {a.shape[1]}, "
                         f"the weight {w.b.shape[1]}")
    if w.smooth is not None and a.dtype != torch.float32:
        raise ValueError("sc_matmul_prepared: a weight prepared with smooth_scales needs a float32 a")
    dev_in = a.device
    if a.is_cuda and a.device != w.device:
        raise ValueError(f"sc_matmul_prepared: a is on {a.device}, the weight on {w.device}")
    with torch.cuda.device(w.device):
        ad = K._to_device(a)
        used = []
        y = K._launch(_lib.PER_ROW, w.mode, ad, w.b, w.sc_prec, w.tables, group_a=group_a,
                      group_b=w.group_b, smooth=w.smooth, workspace=w.workspace, b_ready=w.ready,
                      workspace_out=used)
        w.workspace, w.ready = used[0], True
    return y if dev_in.type == "cuda" else K._to_host(y)
