"""Row-group quantisation (API of scmp_kernels/quant/grouped.py).

Rows come in groups of ``G`` (a final partial group takes the remainder;
``G >= rows`` is one group). Symmetric: ``scale = max(absmax, 1e-5) / q_max``,
``x_int = clamp(round(x / scale), +-q_max)``, sign with 0 -> +1. Asymmetric:
``scale = max(max - min, 1e-5) / q_max``, ``zp = clamp(round(-min / scale),
0, q_max)``, ``x_int = clamp(round(x / scale + zp), 0, q_max)``. The device
kernels compute the same float32 operations as the reference's torch ops.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib


def _dev(x: torch.Tensor) -> torch.Tensor:
    if x.device.type != "cuda":
        _lib.require_cuda()
        x = x.cuda()
    return x.float().contiguous()


def _sym(x: torch.Tensor, batch: int, rows: int, cols: int, G: int, q_max: int):
    dev = x.device
    scale = torch.empty(batch * rows, dtype=torch.float32, device=dev)
    xi = torch.empty(batch * rows, cols, dtype=torch.float32, device=dev)
    sign = torch.empty(batch * rows, cols, dtype=torch.int8, device=dev)
    stats = torch.empty(3 * batch * rows + 1, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().scmp_grouped_symmetric_quant(
            x.data_ptr(), batch, rows, cols, G, q_max, scale.data_ptr(), xi.data_ptr(),
            sign.data_ptr(), stats.data_ptr(), ctypes.c_void_p(_lib.stream_handle(dev))),
            "_grouped_symmetric_quant")
    return scale, xi, sign


def _grouped_symmetric_quant(x: torch.Tensor, G: int, q_max: int):
    """grouped.py:13-75. Returns (scale_row, x_int, sign)."""
    dev_in = x.device
    x = _dev(x)
    rows, cols = x.shape
    s, xi, sg = _sym(x, 1, rows, cols, G, q_max)
    return s.to(dev_in), xi.to(dev_in), sg.to(dev_in)


def _grouped_asymmetric_quant(x: torch.Tensor, G: int, q_max: int):
    """grouped.py:78-133. Returns (scale_row, zp_row, x_int)."""
    dev_in = x.device
    x = _dev(x)
    rows, cols = x.shape
    dev = x.device
    scale = torch.empty(rows, dtype=torch.float32, device=dev)
    zp = torch.empty(rows, dtype=torch.float32, device=dev)
    xi = torch.empty(rows, cols, dtype=torch.float32, device=dev)
    stats = torch.empty(3 * rows + 1, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().scmp_grouped_asymmetric_quant(
            x.data_ptr(), rows, cols, G, q_max, scale.data_ptr(), zp.data_ptr(), xi.data_ptr(),
            stats.data_ptr(), ctypes.c_void_p(_lib.stream_handle(dev))), "_grouped_asymmetric_quant")
    return scale.to(dev_in), zp.to(dev_in), xi.to(dev_in)


def _grouped_symmetric_quant_batched(x: torch.Tensor, G: int, q_max: int):
    """grouped.py:136-163 (G == 1 or G >= rows). Returns scale (BH, rows),
    x_int and sign (BH, rows, cols)."""
    assert x.dim() == 3, f"expected (BH, rows, cols), got {tuple(x.shape)}"
    dev_in = x.device
    x = _dev(x)
    BH, rows, cols = x.shape
    if not (G == 1 or G >= rows):
        raise NotImplementedError(
            f"_grouped_symmetric_quant_batched: G={G} not supported (use G=1 or G>=rows)")
    s, xi, sg = _sym(x, BH, rows, cols, G, q_max)
    return (s.view(BH, rows).to(dev_in), xi.view(BH, rows, cols).to(dev_in),
            sg.view(BH, rows, cols).to(dev_in))


__all__ = ["_grouped_symmetric_quant", "_grouped_asymmetric_quant", "_grouped_symmetric_quant_batched"]
