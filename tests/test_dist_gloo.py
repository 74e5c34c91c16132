"""Multi-process logic of the sharded sc_matmul on CPU (gloo, world size 2).

Each rank holds its row shard of b, computes its column block with the CPU
oracle standing in for the GPU kernel, and the driver in
scmp_kernels_b200.dist all-gathers the blocks. The assembled output must
equal the single-process oracle result bit for bit (per_row, unipolar with
SmoothQuant, chunked, per_tensor with the all-reduced global range, and
per_head sharded by heads). A rank that fails before the collective must
make the other rank's collective fail within the process-group timeout.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback
import zlib

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = {
    "per_row": (dict(granularity="per_row", mode="bipolar", sc_prec=8), (9, 13, 40)),
    "per_row_uni_smooth": (dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64,
                                smooth=True), (7, 11, 33)),
    "chunked": (dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=16, stoc_len=64,
                     rng_levels=64), (6, 9, 40)),
    "per_tensor": (dict(granularity="per_tensor", mode="bipolar", sc_prec=8), (8, 13, 24)),
    "per_tensor_uni_smooth": (dict(granularity="per_tensor", mode="unipolar", sc_prec=6, smooth=True),
                              (5, 7, 20)),
    "per_head": (dict(granularity="per_head", sc_prec=8), (5, 6, 7, 12)),
}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(name):
    kw, shape = CASES[name]
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 1000)
    if name == "per_head":
        bh, n, m, d = shape
        a, b = torch.randn(bh, n, d, generator=g), torch.randn(bh, m, d, generator=g)
    else:
        n, m, d = shape
        a, b = torch.randn(n, d, generator=g), torch.randn(m, d, generator=g) * 0.1
    s = torch.rand(a.shape[-1], generator=g) + 0.5 if kw.get("smooth") else None
    return kw, a, b, s


def _oracle_matmul(a, b, granularity, ranges=None, **kw):
    sys.path.insert(0, REPO)
    from oracle import sc_oracle as O
    s = kw.pop("smooth_scales", None)
    an, bn = a.numpy(), b.numpy()
    if ranges is not None:
        if s is not None:
            an, bn = O.smooth(an, bn, s.numpy())
        L = kw.get("stoc_len") or 2 ** kw["sc_prec"]
        y = O.per_tensor_2d(an, bn, ranges["max_fp_a"], ranges["min_fp_a"], ranges["max_fp_b"],
                            ranges["min_fp_b"], kw.get("mode", "bipolar"), kw["sc_prec"], kw.get("config"),
                            L, kw.get("rng_levels"), env={})
    else:
        y = O.sc_matmul(an, bn, granularity, smooth_scales=None if s is None else s.numpy(), env={}, **kw)
    return torch.from_numpy(np.ascontiguousarray(y))


def _worker(rank, world, port, name, fail_rank, q):
    try:
        sys.path.insert(0, REPO)
        from scmp_kernels_b200 import dist as D
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
        kw, a, b, s = _inputs(name)
        kw = {k: v for k, v in kw.items() if k != "smooth"}
        if s is not None:
            kw["smooth_scales"] = s
        if rank == fail_rank:
            raise RuntimeError("injected failure before the all-gather")
        gran = kw.pop("granularity")
        if gran == "per_head":
            lo, hi = D.shard_bounds(a.shape[0], world, rank)
            y = D.sc_matmul_sharded_heads(a[lo:hi], b[lo:hi], a.shape[0], matmul=_oracle_matmul, **kw)
        else:
            lo, hi = D.shard_bounds(b.shape[0], world, rank)
            y = D.sc_matmul_sharded(a, b[lo:hi].contiguous(), b.shape[0], gran, matmul=_oracle_matmul, **kw)
        q.put((rank, "ok", y.numpy()))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=2)}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(name, fail_rank=-1, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, name, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(world):
        r, status, val = q.get(timeout=120)
        res[r] = (status, val)
    for p in ps:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("name", sorted(CASES))
def test_sharded_equals_single_process(name):
    res = _run(name)
    kw, a, b, s = _inputs(name)
    kw = {k: v for k, v in kw.items() if k != "smooth"}
    gran = kw.pop("granularity")
    if s is not None:
        kw["smooth_scales"] = s
    ref = _oracle_matmul(a, b, gran, **kw).numpy()
    for r, (status, val) in res.items():
        assert status == "ok", val
        assert np.array_equal(val, ref), f"rank {r}: max |diff| {np.abs(val - ref).max()}"


def test_rank_failure_surfaces_on_the_other_rank():
    res = _run("per_row", fail_rank=1)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    assert res[0][0] == "error", "rank 0's all-gather should fail once rank 1 is gone"
