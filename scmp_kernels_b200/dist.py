"""Multi-GPU sc_matmul: the weight operand sharded by rows, outputs all-gathered.

One process per GPU (``torch.distributed``, NCCL). ``a`` (activations) is
replicated on every rank; rank ``r`` holds rows ``shard_bounds(M, W, r)`` of
``b`` (weights), computes its ``(N, M_r)`` column block of ``a @ b.T`` with no
data-path communication, and one all-gather assembles ``(N, M)`` on every
rank. Quantisation of the per_row, chunked and per_head paths is row- (or
head-) local, so every block is bit-identical to the single-GPU result. The
per_tensor path needs b's global range: the ranks all-reduce (MAX / MIN)
their shard's range first and pass the global values down. per_head work is
sharded by heads instead (``shard_heads``).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_bounds(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of ``rank``: equal ceil-sized shards, the last ones short."""
    per = (rows + world - 1) // world
    start = min(rows, rank * per)
    return start, min(rows, start + per)


def _all_gather_cols(y: torch.Tensor, rows_total: int, world: int, group) -> torch.Tensor:
    """All-gather ``(..., N, M_r)`` column blocks (padded to equal width) into ``(..., N, M)``."""
    per = (rows_total + world - 1) // world
    pad = per - y.shape[-1]
    yp = torch.nn.functional.pad(y, (0, pad)) if pad else y.contiguous()
    parts = [torch.empty_like(yp) for _ in range(world)]
    dist.all_gather(parts, yp, group=group)
    return torch.cat(parts, dim=-1)[..., :rows_total]


def sc_matmul_sharded(a: torch.Tensor, b_shard: torch.Tensor, rows_total: int,
                      granularity: str = "per_row", *, group=None,
                      matmul: Optional[Callable] = None, **kw) -> torch.Tensor:
    """``sc_matmul(a, b)`` with ``b`` sharded by rows over the process group.

    a: replicated ``(N, D)`` (or ``(BH, N, D)``); b_shard: this rank's rows of
    b as given by ``shard_bounds(rows_total, world, rank)``; kw: the
    ``sc_matmul`` keyword arguments. ``matmul`` replaces the per-rank compute
    (the default is this package's ``sc_matmul``).
    """
    world = dist.get_world_size(group)
    if granularity == "per_head":
        raise ValueError("sc_matmul_sharded: per_head is sharded by heads, use sc_matmul_sharded_heads")
    if granularity != "per_tensor":
        if matmul is None:
            from .sc.matmul import sc_matmul as matmul
        y = matmul(a, b_shard, granularity, **kw)
        return _all_gather_cols(y, rows_total, world, group)
    # per_tensor: quantisation uses b's global range (of the smoothed operand
    # when smooth_scales is given, as sc_matmul smooths before reducing)
    smooth = kw.get("smooth_scales")
    aa = a / smooth.to(a) if smooth is not None else a
    bs = b_shard * smooth.to(b_shard) if smooth is not None else b_shard
    if bs.numel():
        r = torch.stack([bs.amax(), -bs.amin()]).to(torch.float32)
    else:
        r = torch.full((2,), float("-inf"), device=bs.device)
    dist.all_reduce(r, op=dist.ReduceOp.MAX, group=group)
    ranges = dict(max_fp_a=float(aa.max()), min_fp_a=float(aa.min()),
                  max_fp_b=float(r[0]), min_fp_b=-float(r[1]))
    if matmul is not None:
        y = matmul(a, b_shard, granularity, ranges=ranges, **kw)
    else:
        from .sc.kernels import _sc_matmul_per_tensor
        mode, sc_prec = kw.get("mode", "bipolar"), kw.get("sc_prec", 8)
        stoc_len, rng_levels = kw.get("stoc_len"), kw.get("rng_levels")
        if kw.get("halve_bipolar_stoc_len") and mode == "bipolar":  # matmul.py:177-182
            h = 2 ** (sc_prec - 1)
            stoc_len = h if stoc_len is None else stoc_len
            rng_levels = h if rng_levels is None else rng_levels
        y = _sc_matmul_per_tensor(a, b_shard, **ranges, mode=mode, sc_prec=sc_prec,
                                  config=kw.get("config"), stoc_len=stoc_len, rng_levels=rng_levels,
                                  smooth_scales=smooth)
    return _all_gather_cols(y, rows_total, world, group)


def sc_matmul_sharded_heads(a_shard: torch.Tensor, b_shard: torch.Tensor, heads_total: int, *,
                            group=None, matmul: Optional[Callable] = None, **kw) -> torch.Tensor:
    """per_head work sharded by heads: each rank holds heads
    ``shard_bounds(heads_total, world, rank)`` of both operands; the
    ``(BH_r, N, M)`` results are all-gathered into ``(BH, N, M)``."""
    world = dist.get_world_size(group)
    if matmul is None:
        from .sc.matmul import sc_matmul as matmul
    y = matmul(a_shard, b_shard, "per_head", **kw)
    per = (heads_total + world - 1) // world
    pad = per - y.shape[0]
    yp = torch.nn.functional.pad(y, (0, 0, 0, 0, 0, pad)) if pad else y.contiguous()
    parts = [torch.empty_like(yp) for _ in range(world)]
    dist.all_gather(parts, yp, group=group)
    return torch.cat(parts, dim=0)[:heads_total]
