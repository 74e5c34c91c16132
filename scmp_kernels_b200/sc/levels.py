"""Per-row-group stream lengths in one call: ``sc_matmul_levels``.

The reference composes mixed precision in its caller: rows of the activation
are classified into levels (``classify_rows_by_metric``,
scmp_kernels/mp/config.py:154-191, or the range classifier of :924-1007) and
``sc_matmul`` runs once per level on the gathered rows, with that level's
``stoc_len`` (and, in the fixed-grid mode, ``rng_levels = stoc_len``); the
per-level results are scattered back. ``sc_matmul_levels`` gives the same bits
in one native call (``scmp_sc_matmul_levels``): a's rows are grouped by level
on the device, a is quantised once with every row on its level's grid, b once
per level, and one SC-GEMM launch takes each tile's stream length, b operand
and epilogue scale from its level.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Union

import torch

from .. import _lib
from . import kernels as K


def _grid_of(level: int, L: int, sc_prec: int, rng_levels) -> int:
    if rng_levels is None:
        return 2 ** sc_prec
    if isinstance(rng_levels, str):
        if rng_levels != "stoc_len":
            raise ValueError(f"sc_matmul_levels: rng_levels must be None, 'stoc_len' or a list, got {rng_levels!r}")
        return int(L)
    return int(rng_levels[level])


def _compose(a, b, row_levels, stoc_len_levels, grids, **kw):
    """The reference's composition: one sc_matmul per level on its rows."""
    from .matmul import sc_matmul
    out = torch.empty(a.shape[0], b.shape[0], dtype=torch.float32, device=a.device)
    rl = row_levels.to(a.device)
    for lv, (L, G) in enumerate(zip(stoc_len_levels, grids)):
        rows = torch.nonzero(rl == lv).flatten()
        if rows.numel():
            out[rows] = sc_matmul(a[rows].contiguous(), b, "per_row", stoc_len=L, rng_levels=G, **kw)
    return out


@torch.no_grad()
def sc_matmul_levels(a: torch.Tensor, b: torch.Tensor, row_levels: torch.Tensor,
                     stoc_len_levels: Sequence[int], granularity: str = "per_row", *, mode: str = "bipolar",
                     sc_prec: int = 8, rng_levels: Union[None, str, Sequence[int]] = None, chunk_d: int = 0,
                     group_a: int = 1, group_b: int = 1, config: Optional[dict] = None,
                     smooth_scales: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``sc_matmul`` with a stream length per row of ``a``.

    a: ``(N, D)``; b: ``(M, D)``; row_levels: ``(N,)`` integer level index of
    every row of a (``RowAssignment.row_levels``); stoc_len_levels: the
    stream length of every level (at most four levels). rng_levels: ``None``
    (the grid 2**sc_prec for every level), ``"stoc_len"`` (each level's grid
    is its stream length) or one grid per level. The other arguments are
    sc_matmul's (granularity "per_row" only).

    Returns float32 ``(N, M)``, equal bit for bit to computing the rows of
    each level ``l`` as ``sc_matmul(a[rows_l], b, "per_row",
    stoc_len=stoc_len_levels[l], rng_levels=<grid of l>, ...)``. One native
    call on a B200 (SM pairs, e2m1 operands, padded stream lengths of 64 to
    512, and group_a == 1 unless the chunked path applies); other cases run
    that composition on the GPU.
    """
    if granularity != "per_row":
        raise ValueError(f"sc_matmul_levels: granularity must be 'per_row', got '{granularity}'")
    if mode not in ("bipolar", "unipolar"):
        raise ValueError(f"sc_matmul_levels: unknown mode '{mode}'")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("sc_matmul_levels: 2D operands with the same inner dimension")
    nlev = len(stoc_len_levels)
    if not 1 <= nlev <= _lib.MAX_LEVELS:
        raise ValueError(f"sc_matmul_levels: 1 to {_lib.MAX_LEVELS} levels, got {nlev}")
    if row_levels.dim() != 1 or row_levels.shape[0] != a.shape[0]:
        raise ValueError("sc_matmul_levels: row_levels must hold one level per row of a")
    if chunk_d > 0 and mode != "bipolar":
        raise ValueError(
            f"sc_matmul: chunk_d > 0 requires mode='bipolar', got '{mode}'. "
            f"D-chunking is not implemented for unipolar quantization.")
    grids = [_grid_of(i, L, sc_prec, rng_levels) for i, L in enumerate(stoc_len_levels)]
    D = a.shape[1]
    chunked = mode == "bipolar" and chunk_d > 0 and D > chunk_d
    kw = dict(mode=mode, sc_prec=sc_prec, chunk_d=chunk_d, group_a=group_a, group_b=group_b, config=config,
              smooth_scales=smooth_scales)
    lps = [K._next_pow2(max(32, int(L))) for L in stoc_len_levels]
    native = (not K._FORCE_SIMT and (chunked or group_a == 1) and all(64 <= lp <= 512 for lp in lps)
              and (not chunked or chunk_d % 8 == 0))
    dev_in = a.device
    a_, b_, s = K._prep_smooth(a, b, smooth_scales)
    a_, b_ = K._to_device(a_), K._to_device(b_)
    if not native:
        y = _compose(a_, b_, row_levels, stoc_len_levels, grids, **dict(kw, smooth_scales=(
            None if s is None else smooth_scales)))
        return y if dev_in.type == "cuda" else K._to_host(y)
    dev = a_.device
    cfg = K._default_config(config, chunk_d if chunked else D, sc_prec)
    levels = (_lib.LevelDesc * nlev)()
    keep = []
    for i, (L, G) in enumerate(zip(stoc_len_levels, grids)):
        t = K._get_cached_enable_tables(cfg, sc_prec, dev, int(L), G)
        amap, bmap = t.maps_for(D, chunk_d if chunked else None)
        keep += [t, amap, bmap]
        levels[i] = _lib.LevelDesc(stoc_len=t.L, rng_levels=t.G, vcap=t.vcap, lp=t.lp, ktab=t.ktab.data_ptr(),
                                   pattern4=t.pattern4.data_ptr(), amap=amap.data_ptr(), bmap=bmap.data_ptr())
    n, m = a_.shape[0], b_.shape[0]
    rl = row_levels.to(device=dev, dtype=torch.int32).contiguous()
    redirect = getattr(K._REDIRECT, "value", None)
    out = None
    if redirect is not None:
        peers, n_peers, out_offset, out_ld, out, self_index = redirect
    else:
        out = torch.empty((n, m), dtype=torch.float32, device=dev)
    desc = _lib.MatmulDesc(
        granularity=_lib.PER_ROW, mode=_lib.BIPOLAR if mode == "bipolar" else _lib.UNIPOLAR, sc_prec=sc_prec,
        stoc_len=int(stoc_len_levels[0]), rng_levels=grids[0], chunk_d=chunk_d, group_a=group_a, group_b=group_b,
        batch=1, n=n, m=m, d=D, a=a_.data_ptr(), b=b_.data_ptr(),
        smooth_scales=s.data_ptr() if s is not None else None, out=out.data_ptr())
    if redirect is not None:
        desc.out = None
        desc.out_peers = ctypes.cast(peers, ctypes.c_void_p)
        desc.n_out_peers, desc.out_offset, desc.out_ld = n_peers, out_offset, out_ld
        desc.out_self = self_index + 1
    L_ = _lib.lib()
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(L_.scmp_sc_matmul_levels_workspace_size(ctypes.byref(desc), levels, nlev, ctypes.byref(ws_bytes)),
               "sc_matmul_levels")
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=dev)
    _lib.check(L_.scmp_sc_matmul_levels(ctypes.byref(desc), levels, nlev, ctypes.c_void_p(rl.data_ptr()),
                                        ctypes.c_void_p(ws.data_ptr()), ws_bytes.value,
                                        ctypes.c_void_p(_lib.stream_handle(dev))), "sc_matmul_levels")
    return out if dev_in.type == "cuda" else K._to_host(out)
