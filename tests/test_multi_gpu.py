"""The sharded sc_matmul on two or more GPUs (NCCL, one process per GPU).

The fused path (each rank's GEMM epilogue stores its column block, or its
heads, straight into every rank's output buffer over NVLink) and the gathered
path (NCCL all-gather after the GEMM) must both equal the single-GPU result
bit for bit, for per_row, per_tensor (global ranges all-reduced) and per_head
sharded by heads, over several calls in a row (the two alternating buffers).
Skipped on a machine with fewer than two GPUs.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu
if torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs", allow_module_level=True)

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(kind):
    g = torch.Generator().manual_seed({"per_row": 1, "per_tensor": 2, "per_head": 3}[kind])
    if kind == "per_head":
        return torch.randn(6, 70, 64, generator=g), torch.randn(6, 90, 64, generator=g)
    return torch.randn(300, 512, generator=g), torch.randn(1000, 512, generator=g) * 0.05


def _worker(rank, port, q):
    try:
        sys.path.insert(0, REPO)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from scmp_kernels_b200 import sc_matmul
        from scmp_kernels_b200 import dist as SD
        res = {}
        for kind in ("per_row", "per_tensor", "per_head"):
            a, b = (x.to(dev) for x in _inputs(kind))
            ref = sc_matmul(a, b, kind, sc_prec=8)
            if kind == "per_head":
                h0, h1 = SD.shard_bounds(a.shape[0], WORLD, rank)
                run = lambda fused: SD.sc_matmul_sharded_heads(a[h0:h1], b[h0:h1], a.shape[0], sc_prec=8,
                                                               fused=fused)
            else:
                lo, hi = SD.shard_bounds(b.shape[0], WORLD, rank)
                bs = b[lo:hi].contiguous()
                run = lambda fused: SD.sc_matmul_sharded(a, bs, b.shape[0], kind, sc_prec=8, fused=fused)
            ok = all(torch.equal(run(True), ref) for _ in range(3)) and torch.equal(run(False), ref)
            res[kind] = ok
        SD.release_peer_buffers()
        q.put((rank, "ok", res))
    except Exception as e:
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc(limit=3)}"))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_sharded_fused_and_gathered_equal_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    out = [q.get(timeout=600) for _ in range(WORLD)]
    for p in ps:
        p.join(timeout=120)
    for rank, status, val in out:
        assert status == "ok", val
        assert all(val.values()), f"rank {rank}: {val}"


@pytest.mark.parametrize("granularity,chunk_d,shape", [
    ("per_tensor", 0, "2d"),
    ("per_row", 0, "2d"),
    ("per_row", 128, "2d"),
    ("per_row", 0, "3d"),
    ("per_head", 0, "3d"),
    ("per_row", 0, "2d_long"),
])
def test_runs_on_second_gpu(granularity, chunk_d, shape):
    """One process, two devices (the reference's multi-GPU device guard,
    tests/test_sc_smoke.py:139-172): inputs on cuda:1 with cuda:0 current run
    on cuda:1, leave cuda:0 current and equal the cuda:0 result. The "2d_long"
    case launches the wide-tile GEMM (over 48 KB of shared memory, a per-device
    kernel attribute) on cuda:0, then cuda:1, then cuda:0 again."""
    sys.path.insert(0, REPO)
    from scmp_kernels_b200 import sc_matmul
    torch.manual_seed(0)
    if shape == "2d":
        a0, b0 = torch.randn(8, 256, device="cuda:0"), torch.randn(16, 256, device="cuda:0")
    elif shape == "2d_long":
        a0, b0 = torch.randn(300, 1000, device="cuda:0"), torch.randn(520, 1000, device="cuda:0")
    else:
        a0, b0 = torch.randn(4, 8, 64, device="cuda:0"), torch.randn(4, 16, 64, device="cuda:0")
    torch.cuda.set_device(0)
    y0 = sc_matmul(a0, b0, granularity=granularity, chunk_d=chunk_d, sc_prec=8)
    y1 = sc_matmul(a0.to("cuda:1"), b0.to("cuda:1"), granularity=granularity, chunk_d=chunk_d, sc_prec=8)
    y2 = sc_matmul(a0, b0, granularity=granularity, chunk_d=chunk_d, sc_prec=8)
    assert y1.device.index == 1
    assert torch.cuda.current_device() == 0
    assert torch.equal(y0.cpu(), y1.cpu()) and torch.equal(y0, y2)
