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
        if a.dim() == 2:
            def per_row_2d(x, y):
                if chunk_d > 0:
                    return _sc_matmul_per_row_mlp(x, y, mode=mode, group_a=group_a, group_b=group_b,
                                                  chunk_d=chunk_d, **kw)
                return _sc_matmul_per_row(x, y, group_a=group_a, group_b=group_b, mode=mode, **kw)
            if _host_pipelined_applies(a, b):
                if smooth_scales is not None and smooth_scales.device.type != "cuda":
                    # on the device before the operands' copies are queued:
                    # host-to-device copies run in the order they are issued,
                    # so a copy issued inside the first block's call would wait
                    # for all of a's and b's (config 5: first GEMM at 22 ms
                    # instead of 5.5 ms)
                    kw["smooth_scales"] = smooth_scales.to(torch.device("cuda", torch.cuda.current_device()))
                L = stoc_len if stoc_len is not None else 2 ** sc_prec
                return _per_row_host_pipelined(a, b, per_row_2d, group_a, group_b, L)
            return per_row_2d(a, b)
        return _sc_matmul_per_row_batched(a, b, group_a=group_a, group_b=group_b, mode=mode, **kw)
    return _sc_matmul_per_head_bipolar(a, b, **kw)


# Host operands: the rows of a are processed in three blocks. The first block
# runs against b's row blocks as they arrive (b is copied to the device block
# by block on a copy stream while the previous block computes); the later
# blocks run against the whole of b (the middle one is one call, so that
# fewer, larger GEMMs run; the last one is a third of the rest, so that little
# result is left to copy back after the last GEMM). Each finished block of
# result rows (contiguous in memory) is copied back on a second copy stream
# while the next block computes. The first block is sized so that its GEMM
# against one b block takes about as long as that block's copy: r rows against
# c rows of b cost 2*r*c*D*L tensor ops (about 6.5e15 per s) and the copy
# 4*c*D bytes (about 55e9 per s), equal at r = 2^18 / L rows (1024 at L = 256,
# a quarter of config 2's a; 4096 at L = 64, half of config 5's), at least a
# quarter and at most half of a, in whole 256-row tiles. Applies to 2D per_row
# calls with both operands in pinned host memory and a CUDA device present;
# per_row quantisation is row-local (row groups are kept whole), so the blocks
# give the same bits as one call.
_HOST_FIRST_ROWS_L = 1 << 18  # first block's rows times the stream length
_HOST_B_BLOCKS = 4            # blocks of b's rows in the first pass
_HOST_MIN_ROWS = 1024         # smaller calls are not split


def _host_pipelined_applies(a: torch.Tensor, b: torch.Tensor) -> bool:
    return (a.device.type == "cpu" and b.device.type == "cpu" and torch.cuda.is_available()
            and a.is_pinned() and b.is_pinned() and a.shape[0] >= _HOST_MIN_ROWS
            and b.shape[0] >= _HOST_MIN_ROWS)


def _blocks(total: int, step: int, unit: int):
    step = max(1, (step + unit - 1) // unit) * unit  # whole row groups
    return [(r, min(total, r + step)) for r in range(0, total, step)]


def _a_blocks(n: int, L: int, group_a: int):
    """Row ranges of a's blocks (first, middle, last); inner boundaries on
    whole row groups."""
    tile = 256

    def up(x, k):
        return -(-x // k) * k

    first = up(max(1, _HOST_FIRST_ROWS_L // max(1, L)), tile)
    first = up(min(max(first, (n + 3) // 4), (n + 1) // 2), group_a)
    if first >= n:
        return [(0, n)]
    b2 = up(n - up((n - first) // 3, tile), group_a)  # start of the last block
    if b2 <= first or b2 >= n:
        return [(0, first), (first, n)]
    return [(0, first), (first, b2), (b2, n)]


def _per_row_host_pipelined(a: torch.Tensor, b: torch.Tensor, run, group_a: int, group_b: int,
                            L: int = 256) -> torch.Tensor:
    from . import kernels as K
    dev = torch.device("cuda", torch.cuda.current_device())
    n, m = a.shape[0], b.shape[0]
    a_blocks = _a_blocks(n, L, group_a)
    b_blocks = _blocks(m, (m + _HOST_B_BLOCKS - 1) // _HOST_B_BLOCKS, group_b)
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    a_f = a if a.dtype == torch.float32 else a.float()
    b_f = b if b.dtype == torch.float32 else b.float()
    a_dev = torch.empty(a_f.shape, dtype=torch.float32, device=dev)
    b_dev = torch.empty(b_f.shape, dtype=torch.float32, device=dev)
    out_dev = torch.empty((n, m), dtype=torch.float32, device=dev)
    out_host = torch.empty((n, m), dtype=torch.float32, pin_memory=True)
    for t, st in ((a_dev, comp), (b_dev, comp), (out_dev, s_out)):
        t.record_stream(st)
    # The staging buffers come from the caller's stream's pool: a block freed
    # there may still be in use by work queued on it, so the copy stream
    # starts after that work.
    s_in.wait_stream(comp)
    # copies in the order they are needed: a's first block, b's blocks, a's other blocks
    ev_b = []
    with torch.cuda.stream(s_in):
        r0, r1 = a_blocks[0]
        a_dev[r0:r1].copy_(a_f[r0:r1], non_blocking=True)
        for c0, c1 in b_blocks:
            b_dev[c0:c1].copy_(b_f[c0:c1], non_blocking=True)
            ev_b.append(torch.cuda.Event())
            ev_b[-1].record(s_in)
        ev_a = [None]
        for r0, r1 in a_blocks[1:]:
            a_dev[r0:r1].copy_(a_f[r0:r1], non_blocking=True)
            ev_a.append(torch.cuda.Event())
            ev_a[-1].record(s_in)
    for i, (r0, r1) in enumerate(a_blocks):
        if i == 0:
            for (c0, c1), ev in zip(b_blocks, ev_b):
                comp.wait_event(ev)
                with K.output_to([out_dev.data_ptr()], c0, m, out_dev):
                    run(a_dev[r0:r1], b_dev[c0:c1])
        else:
            comp.wait_event(ev_a[i])
            with K.output_to([out_dev.data_ptr()], r0 * m, m, out_dev):
                run(a_dev[r0:r1], b_dev)
        s_out.wait_stream(comp)
        with torch.cuda.stream(s_out):
            out_host[r0:r1].copy_(out_dev[r0:r1], non_blocking=True)
    s_out.synchronize()
    return out_host
