"""Seeded synthetic inputs for the five benchmark configurations of ``sc_matmul``.

The reference publishes no input tensors for its headline shapes (its accuracy
benchmarks capture Llama activations that are not shipped), so these recipes
stand in for them with the shapes and value distributions the benchmark
configurations name:

  1. per_tensor bipolar, a 64x256 and b 32x256, iid N(0,1) from one generator.
  2. per_row bipolar at the Llama-7B MLP up-projection: a 4096x4096 N(0,1) with
     1% of the channels scaled x20 (outliers), b 11008x4096 N(0, 0.02^2).
  3. per_head bipolar ViT-B/16 attention, BH=768: q, k 768x197x64 N(0,1); the
     softmax.V pass multiplies row-softmax(N(0,1) logits) 768x197x197 by
     V^T 768x64x197.
  4. per_row bipolar chunk_d=64 at ViT-B fc2: a = GELU(N(0,1)) 12608x3072,
     b 768x3072 N(0, 0.02^2); row groups of 4 are assigned stoc_len in
     {256, 128, 64} by the tercile of their value range (caller-side policy).
  5. per_row unipolar with SmoothQuant at the Llama-70B MLP: a 8192x8192 with
     outlier channels as in 2, b 28672x8192 N(0, 0.015^2), per-channel smooth
     scales with alpha = 0.5.

Every tensor comes from one ``torch.Generator`` seeded per configuration, drawn
in a fixed order, so a recipe reproduces bit-identical inputs on any machine
when generated on the CPU.
"""
from __future__ import annotations

from typing import Optional

import torch


def _gen(seed: int, device: str) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def outlier_activations(rows: int, cols: int, g: torch.Generator, device: str,
                        frac: float = 0.01, factor: float = 20.0) -> torch.Tensor:
    """N(0,1) activations with ``round(frac*cols)`` channels scaled by ``factor``."""
    a = torch.randn(rows, cols, generator=g, device=device)
    n_out = max(1, int(cols * frac))
    ch = torch.randperm(cols, generator=g, device=device)[:n_out]
    a[:, ch] *= factor
    return a


def config1(device: str = "cpu"):
    g = _gen(0, device)
    a = torch.randn(64, 256, generator=g, device=device)
    b = torch.randn(32, 256, generator=g, device=device)
    return a, b


def config2(device: str = "cpu", n: int = 4096, m: int = 11008, d: int = 4096):
    g = _gen(2, device)
    a = outlier_activations(n, d, g, device)
    b = torch.randn(m, d, generator=g, device=device) * 0.02
    return a, b


def config3(device: str = "cpu", bh: int = 768, n: int = 197, d: int = 64):
    """Returns (q, k, probs, v_t) for the QK and softmax.V passes."""
    g = _gen(3, device)
    q = torch.randn(bh, n, d, generator=g, device=device)
    k = torch.randn(bh, n, d, generator=g, device=device)
    logits = torch.randn(bh, n, n, generator=g, device=device)
    probs = torch.softmax(logits, dim=-1)
    v_t = torch.randn(bh, d, n, generator=g, device=device)
    return q, k, probs, v_t


def config4(device: str = "cpu", n: int = 12608, m: int = 768, d: int = 3072):
    g = _gen(4, device)
    a = torch.nn.functional.gelu(torch.randn(n, d, generator=g, device=device))
    b = torch.randn(m, d, generator=g, device=device) * 0.02
    return a, b


def config5(device: str = "cpu", n: int = 8192, m: int = 28672, d: int = 8192,
            with_scales: bool = True):
    """Returns (a, b, smooth_scales); scales use alpha = 0.5 on the full tensors."""
    g = _gen(5, device)
    a = outlier_activations(n, d, g, device)
    b = torch.randn(m, d, generator=g, device=device) * 0.015
    s: Optional[torch.Tensor] = None
    if with_scales:
        from .quant.smoothquant import accumulate_act_scales, compute_smooth_scales
        s = compute_smooth_scales(accumulate_act_scales(a), b, alpha=0.5)
    return a, b, s


def mp_row_levels(a: torch.Tensor, group: int = 4,
                  levels=(256, 128, 64)) -> dict:
    """Caller-side mixed precision for configuration 4.

    Rows are taken in groups of ``group``; each group's metric is its value
    range (max - min). Groups are ranked by the metric and split into equal
    fractions, the top fraction getting the longest stream, following the
    quantile bucketing of the reference's ``classify_rows_by_metric``
    (scmp_kernels/mp/config.py:154-191). Returns ``{stoc_len: row indices}``.
    """
    rows = a.shape[0]
    n_groups = rows // group
    ag = a[: n_groups * group].reshape(n_groups, group, -1)
    metric = ag.amax(dim=(1, 2)) - ag.amin(dim=(1, 2))
    order = metric.argsort(descending=True)
    out = {}
    offset = 0
    for i, sl in enumerate(levels):
        if i < len(levels) - 1:
            count = round(n_groups / len(levels))
        else:
            count = n_groups - offset
        count = max(0, min(count, n_groups - offset))
        grp = order[offset:offset + count]
        r = (grp[:, None] * group + torch.arange(group, device=a.device)[None, :]).reshape(-1)
        out[sl] = torch.sort(r).values
        offset += count
    if rows % group:
        # a trailing partial group rides with the lowest level
        tail = torch.arange(n_groups * group, rows, device=a.device)
        out[levels[-1]] = torch.cat([out[levels[-1]], tail])
    return out


def mp_row_level_index(a: torch.Tensor, group: int = 4, levels=(256, 128, 64)):
    """The assignment of ``mp_row_levels`` as ``(row_levels, stoc_len_levels)``:
    the level index of every row of a (int32, on a's device; the form of the
    reference's ``RowAssignment.row_levels``) and the stream length of every
    level, the arguments of ``sc_matmul_levels``."""
    lv = mp_row_levels(a, group, levels)
    rl = torch.empty(a.shape[0], dtype=torch.int32, device=a.device)
    for i, L in enumerate(levels):
        rl[lv[L]] = i
    return rl, [int(L) for L in levels]
