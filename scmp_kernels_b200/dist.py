"""Multi-GPU sc_matmul: the weight operand sharded by rows, outputs all-gathered.

One process per GPU (``torch.distributed``). ``a`` (activations) is replicated
on every rank; rank ``r`` holds rows ``shard_bounds(M, W, r)`` of ``b``
(weights) and computes its ``(N, M_r)`` column block of ``a @ b.T`` with no
data-path communication. Quantisation of the per_row, chunked and per_head
paths is row- (or head-) local, so every block is bit-identical to the
single-GPU result; per_tensor needs b's global range, so the ranks all-reduce
(MAX / MIN) their shard's range first and pass the global values down.
per_head work is sharded by heads instead (``sc_matmul_sharded_heads``).

The blocks are assembled in one of two ways:

* fused (NCCL groups of up to 8 ranks on one node, the default there): every
  rank's GEMM epilogue stores its block straight into every rank's full
  output buffer over NVLink (buffers shared with CUDA IPC, kept per output
  shape, two per shape used alternately), then one small NCCL all-reduce
  serves as the barrier after which all blocks have landed;
* gathered: an NCCL (or gloo) all-gather of the blocks after the GEMM.
"""
from __future__ import annotations

import atexit
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib


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


class _DeviceView:
    """``__cuda_array_interface__`` of a float32 buffer owned by the library."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class _PeerOutputs:
    """Two full-output buffers per rank, each mapped into every rank of the
    group. Slots alternate between calls: a rank overwrites slot s of its
    peers only after the barrier of the following call, by which time every
    rank has copied its result out of slot s."""

    def __init__(self, shape, device: torch.device, group):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        nbytes = 4
        for x in shape:
            nbytes *= int(x)
        self.own, self.opened, self.slots = [], [], []
        with torch.cuda.device(device):
            for _ in range(2):
                ptr, handle = _lib.peer_alloc(max(nbytes, 4))
                self.own.append(ptr)
                handles = [None] * self.world
                dist.all_gather_object(handles, handle, group=group)
                ptrs = []
                for r, h in enumerate(handles):
                    if r == self.rank:
                        ptrs.append(ptr)
                    else:
                        q = _lib.peer_open(h)
                        self.opened.append(q)
                        ptrs.append(q)
                view = torch.as_tensor(_DeviceView(ptr, shape), device=device)
                self.slots.append((view, ptrs))
        self.next = 0

    def take(self):
        slot = self.slots[self.next]
        self.next ^= 1
        return slot

    def release(self):
        L = _lib.lib()
        for q in self.opened:
            L.scmp_peer_close(q)
        for p in self.own:
            L.scmp_peer_free(p)
        self.own, self.opened, self.slots = [], [], []


# Buffers per (group members and backend, output shape, device). Keyed by the
# members rather than the group object, so that a group destroyed and another
# created in its place (possibly at the same address) never inherits mappings
# made for different ranks; groups with the same members share the buffers,
# which is safe because every call ends with a barrier over those members.
_PEER_OUTPUTS: dict = {}


def _group_key(group):
    return (tuple(dist.get_process_group_ranks(group if group is not None else dist.group.WORLD)),
            str(dist.get_backend(group)))


def release_peer_buffers(group=None) -> None:
    """Free the fused all-gather buffers (collective: call on every rank,
    after the last sharded call, before destroying the process group)."""
    if _PEER_OUTPUTS:
        dist.barrier(group=group)
    for po in _PEER_OUTPUTS.values():
        po.release()
    _PEER_OUTPUTS.clear()


@atexit.register
def _release_at_exit():  # unmap and free without a collective; the processes are ending
    for po in _PEER_OUTPUTS.values():
        try:
            po.release()
        except Exception:
            pass
    _PEER_OUTPUTS.clear()


def _use_fused(a: torch.Tensor, group, world: int, matmul) -> bool:
    return (matmul is None and 1 < world <= _lib.MAX_OUT_PEERS and a.is_cuda
            and dist.get_backend(group) == "nccl")


def _fused(a, shape, offset: int, ld: int, group, compute, copy: bool = True):
    """Run ``compute()`` with its result scattered into every rank's buffer of
    ``shape`` at ``offset`` / ``ld``; return this rank's copy of the full result
    (with ``copy=False`` the library's buffer itself, see sc_matmul_sharded)."""
    from .sc import kernels as K
    key = (_group_key(group), tuple(shape), a.device.index)
    po = _PEER_OUTPUTS.get(key)
    if po is None:
        po = _PEER_OUTPUTS[key] = _PeerOutputs(shape, a.device, group)
    view, ptrs = po.take()
    with K.output_to(ptrs, offset, ld, view, self_index=po.rank):
        compute()
    # every rank's epilogue has stored its block once this collective completes
    dist.all_reduce(torch.zeros(1, device=a.device), group=group)
    return view.clone() if copy else view


def _collective_device(group, like: torch.Tensor) -> torch.device:
    """Where a small tensor for a collective of ``group`` must live."""
    if dist.get_backend(group) == "nccl":
        return like.device if like.is_cuda else torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def sc_matmul_sharded(a: torch.Tensor, b_shard: torch.Tensor, rows_total: int,
                      granularity: str = "per_row", *, group=None,
                      matmul: Optional[Callable] = None, fused: Optional[bool] = None,
                      gather: bool = True, copy: bool = True, **kw) -> torch.Tensor:
    """``sc_matmul(a, b)`` with ``b`` sharded by rows over the process group.

    a: replicated ``(N, D)`` (or ``(BH, N, D)``); b_shard: this rank's rows of
    b as given by ``shard_bounds(rows_total, world, rank)``; kw: the
    ``sc_matmul`` keyword arguments. ``matmul`` replaces the per-rank compute
    (the default is this package's ``sc_matmul``); ``fused`` selects the
    epilogue all-gather (default: NCCL groups of up to 8 ranks).

    gather=False returns only this rank's ``(..., N, M_r)`` column block, with
    no all-gather (the output stays sharded, as a tensor-parallel consumer
    takes it); operands in pinned host memory then take sc_matmul's streamed
    host path and the block comes back in pinned host memory.

    copy=False (fused path) returns the library's gather buffer itself
    instead of a copy: it holds the result until the second-next fused call
    of the same output shape on this group overwrites it.
    """
    world = dist.get_world_size(group)
    if granularity == "per_head":
        raise ValueError("sc_matmul_sharded: per_head is sharded by heads, use sc_matmul_sharded_heads")
    if fused is None:
        fused = gather and _use_fused(a, group, world, matmul)
    ranges = None
    if granularity == "per_tensor":
        # quantisation uses b's global range (of the smoothed operand when
        # smooth_scales is given, as sc_matmul smooths before reducing)
        smooth = kw.get("smooth_scales")
        aa = a / smooth.to(a) if smooth is not None else a
        bs = b_shard * smooth.to(b_shard) if smooth is not None else b_shard
        if bs.numel():
            r = torch.stack([bs.amax(), -bs.amin()]).to(torch.float32)
        else:
            r = torch.full((2,), float("-inf"), device=bs.device)
        r = r.to(_collective_device(group, bs))
        dist.all_reduce(r, op=dist.ReduceOp.MAX, group=group)
        ranges = dict(max_fp_a=float(aa.max()), min_fp_a=float(aa.min()),
                      max_fp_b=float(r[0]), min_fp_b=-float(r[1]))

    def compute():
        if ranges is None:
            mm = matmul
            if mm is None:
                if "row_levels" in kw:  # a stream length per row of a: sc_matmul_levels
                    from .sc.levels import sc_matmul_levels as mm
                else:
                    from .sc.matmul import sc_matmul as mm
            return mm(a, b_shard, granularity, **kw)
        if matmul is not None:
            return matmul(a, b_shard, granularity, ranges=ranges, **kw)
        from .sc.kernels import _sc_matmul_per_tensor
        mode, sc_prec = kw.get("mode", "bipolar"), kw.get("sc_prec", 8)
        stoc_len, rng_levels = kw.get("stoc_len"), kw.get("rng_levels")
        if kw.get("halve_bipolar_stoc_len") and mode == "bipolar":  # matmul.py:177-182
            h = 2 ** (sc_prec - 1)
            stoc_len = h if stoc_len is None else stoc_len
            rng_levels = h if rng_levels is None else rng_levels
        return _sc_matmul_per_tensor(a, b_shard, **ranges, mode=mode, sc_prec=sc_prec,
                                     config=kw.get("config"), stoc_len=stoc_len, rng_levels=rng_levels,
                                     smooth_scales=kw.get("smooth_scales"))

    if not gather:
        return compute()
    if not fused:
        return _all_gather_cols(compute(), rows_total, world, group)
    rank = dist.get_rank(group)
    lo, hi = shard_bounds(rows_total, world, rank)
    if b_shard.shape[-2] != hi - lo:
        raise ValueError(f"sc_matmul_sharded: rank {rank} holds {b_shard.shape[-2]} rows of b, "
                         f"shard_bounds gives {hi - lo}")
    return _fused(a, (*a.shape[:-1], rows_total), lo, rows_total, group, compute, copy)


def sc_matmul_sharded_heads(a_shard: torch.Tensor, b_shard: torch.Tensor, heads_total: int, *,
                            group=None, matmul: Optional[Callable] = None, fused: Optional[bool] = None,
                            **kw) -> torch.Tensor:
    """per_head work sharded by heads: each rank holds heads
    ``shard_bounds(heads_total, world, rank)`` of both operands; the
    ``(BH_r, N, M)`` results are assembled into ``(BH, N, M)``."""
    world = dist.get_world_size(group)
    if fused is None:
        fused = _use_fused(a_shard, group, world, matmul)
    mm = matmul
    if mm is None:
        from .sc.matmul import sc_matmul as mm

    def compute():
        return mm(a_shard, b_shard, "per_head", **kw)

    if fused:
        rank = dist.get_rank(group)
        h0, h1 = shard_bounds(heads_total, world, rank)
        if a_shard.shape[0] != h1 - h0:
            raise ValueError(f"sc_matmul_sharded_heads: rank {rank} holds {a_shard.shape[0]} heads, "
                             f"shard_bounds gives {h1 - h0}")
        n, m = a_shard.shape[1], b_shard.shape[1]
        return _fused(a_shard, (heads_total, n, m), h0 * n * m, m, group, compute)
    y = compute()
    per = (heads_total + world - 1) // world
    pad = per - y.shape[0]
    yp = torch.nn.functional.pad(y, (0, 0, 0, 0, 0, pad)) if pad else y.contiguous()
    parts = [torch.empty_like(yp) for _ in range(world)]
    dist.all_gather(parts, yp, group=group)
    return torch.cat(parts, dim=0)[:heads_total]
