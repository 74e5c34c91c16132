"""Benchmark of the B200 stochastic-computing matmul (one JSON line on rank 0).

python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config2|config5|config3qk|config3av|config4]
                [--impl ours|reference]

Metric: equivalent SC-GEMM throughput, 2*BH*N*M*D / t, in GOPS (the
reference's headline). A step is one sc_matmul over the workload's resident
operands. At N > 1 the weight operand b is sharded by rows over the ranks and
the output column blocks are all-gathered with NCCL (strong scaling: the job's
total work is fixed). `value` is device-timed (CUDA events, max over ranks);
`e2e` times the public API end to end from pinned host buffers (inputs copied
host->device and the output read back every step). `--impl reference` times
the CPU oracle port of the reference's algorithm on a bounded sample of the
same workload with all host threads (the reference itself is Python + Triton
and only runs on the CPU under its interpreter, which the oracle restates).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

WORKLOADS = {
    # name: (description, builder)
    "config2": "per_row bipolar, Llama-7B MLP up-proj: a 4096x4096, b 11008x4096, p=8, L=256",
    "config5": "per_row unipolar + SmoothQuant, Llama-70B MLP: a 8192x8192, b 28672x8192, p=6, L=64",
    "config3qk": "per_head bipolar ViT-B/16 QK: 768 x (197x64) x (197x64), p=8, L=256",
    "config3av": "per_head bipolar ViT-B/16 softmax.V: 768 x (197x197) x (64x197), p=8, L=256",
    "config4": "per_row bipolar chunk_d=64 ViT-B fc2: a 12608x3072, b 768x3072, p=8, L=256/128/64 by row-range tercile",
}


# DRAM bytes of one GEMM launch (DRAM read + write bytes) from an ncu capture of
# the 2048-row case of the config-2 recipe (395.7 MB,
# profiles/gemm_tc_pair_e2m1_wide480_2048x11008x4096.md), scaled to the 4096
# rows of the full workload: the a rows, the output and the bands of a that
# re-read b all double.
GEMM_TRAFFIC_BYTES = {"config2": 2 * 395.7e6}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="config2", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shape", default=None,
                    help="N,M,D override of the config2/config5 recipes (smaller cases for profiling)")
    return ap.parse_args()


def build_workload(name, device, shape=None):
    """Returns (a, b, kwargs, bh_n_m_d, L, label, calls) with calls = list of
    (a_rows_index or None, kwargs) for workloads composed of several calls."""
    from scmp_kernels_b200 import workloads as W
    if name == "config2":
        n, m, d = shape or (4096, 11008, 4096)
        a, b = W.config2(device, n, m, d)
        return a, b, None, dict(granularity="per_row", mode="bipolar", sc_prec=8), (1, n, m, d), 256
    if name == "config5":
        n, m, d = shape or (8192, 28672, 8192)
        a, b, s = W.config5(device, n, m, d)
        return a, b, s, dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64), \
            (1, n, m, d), 64
    if name in ("config3qk", "config3av"):
        q, k, probs, v_t = W.config3(device)
        if name == "config3qk":
            return q, k, None, dict(granularity="per_head", sc_prec=8), (768, 197, 197, 64), 256
        return probs, v_t, None, dict(granularity="per_head", sc_prec=8), (768, 197, 64, 197), 256
    if name == "config4":
        a, b = W.config4(device)
        return a, b, None, dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=64, group_a=4,
                                group_b=4), (1, 12608, 768, 3072), None
    raise ValueError(name)


def clocks_start(idx):
    f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        p = subprocess.Popen(["nvidia-smi", f"--id={idx}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                              "-lms", "200"], stdout=f, stderr=subprocess.DEVNULL)
    except OSError:
        p = None
    return p, f.name


def clocks_wait_first_sample(path, timeout_s=10.0):
    """Block until the sampler has written its first line, so that its start-up
    (NVML initialisation) happens before the timed region, not inside it."""
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        try:
            if os.path.getsize(path) > 0:
                return
        except OSError:
            pass
        time.sleep(0.05)


def clocks_stop(p, path):
    if p is None:
        return None
    p.terminate()
    try:
        p.wait(timeout=5)
    except subprocess.TimeoutExpired:
        p.kill()
    sms, mx, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in open(path):
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sms.append(float(f[1]))
            mx = float(f[2])
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    os.unlink(path)
    if not sms:
        return None
    load = [s for s in sms if mx and s > 0.5 * mx] or sms
    return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons),
            "samples": len(sms)}


def cpu_baseline(workload, max_seconds=20.0):
    """Time the oracle port (test infrastructure, used only as this baseline)
    on a bounded row sample of the workload; returns the baseline dict."""
    import numpy as np
    import torch
    from oracle import sc_oracle as O
    from scmp_kernels_b200 import workloads as W
    threads = os.cpu_count() or 1
    try:
        from oracle import c_oracle as CO
        have_c = CO.available()
    except Exception:
        have_c = False
    g = torch.Generator().manual_seed(0)
    if workload == "config5":
        a, b = W.outlier_activations(1024, 8192, g, "cpu"), torch.randn(1024, 8192, generator=g) * 0.015
        p, L, D = dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64), 64, 8192
    elif workload.startswith("config3"):
        a, b = torch.randn(16, 197, 64, generator=g), torch.randn(16, 197, 64, generator=g)
        p, L, D = dict(granularity="per_head", sc_prec=8), 256, 64
    else:
        a, b = W.outlier_activations(1024, 4096, g, "cpu"), torch.randn(1024, 4096, generator=g) * 0.02
        p, L, D = dict(granularity="per_row", mode="bipolar", sc_prec=8), 256, 4096
    an, bn = a.numpy(), b.numpy()
    q = dict(p)
    gran = q.pop("granularity")
    rows = 8
    while True:
        sa, sb = np.ascontiguousarray(an[..., :rows, :]), np.ascontiguousarray(bn[..., :rows, :])
        t0 = time.perf_counter()
        if have_c:
            CO.sc_matmul(sa, sb, gran, threads=threads, **q)
        else:
            O.sc_matmul(sa, sb, gran, env={}, **q)
        dt = time.perf_counter() - t0
        if dt > max_seconds / 4 or rows >= an.shape[-2]:
            break
        rows = min(an.shape[-2], rows * 2)
    bh = a.shape[0] if a.dim() == 3 else 1
    ops = 2.0 * bh * rows * rows * D
    return {"value": ops / dt / 1e9, "unit": "GOPS", "cores": threads if have_c else 1,
            "kind": "port", "sample": f"{gran} {workload} slice: {bh}x{rows}x{rows}x{D} (L={L}) in {dt:.2f}s, "
                                      f"{'C oracle, OpenMP' if have_c else 'numpy oracle, 1 thread'}"}


def run_reference(args, rank, world):
    """--impl reference: the oracle port on the host cores, rank 0 only."""
    if rank != 0:
        return
    base = cpu_baseline(args.workload, max_seconds=max(5.0, 60.0 / max(1, args.steps + args.warmup)))
    line = {"metric": "SC-GEMM equiv GOPS (2*BH*N*M*D/s)", "value": base["value"], "unit": "GOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "impl": "reference", "scaling": "strong", "vs_baseline": None, "dtype": "int32-accumulate",
            "data": "synthetic (seeded, reference shapes and distributions)",
            "config": {"workload": args.workload, "desc": WORKLOADS[args.workload]},
            "cpu_baseline": base, "e2e": {"value": base["value"], "unit": "GOPS",
                                          "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    from scmp_kernels_b200 import _lib, sc_matmul

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    shape = tuple(int(x) for x in args.shape.split(",")) if args.shape else None
    a, b, s, kw, (BH, N, M, D), L = build_workload(args.workload, dev, shape)
    # shard the weight operand by rows
    if world > 1:
        rows = b.shape[-2]
        per = (rows + world - 1) // world
        b = b[..., rank * per:min(rows, (rank + 1) * per), :].contiguous()
    kw = dict(kw)
    if s is not None:
        kw["smooth_scales"] = s
    calls = [(None, kw)]
    if args.workload == "config4":
        from scmp_kernels_b200 import workloads as W
        lv = W.mp_row_levels(a, 4, (256, 128, 64))
        calls = [(rows_.to(dev), dict(kw, stoc_len=Lv, rng_levels=Lv)) for Lv, rows_ in lv.items()]
    a_parts = [a if idx is None else a[idx].contiguous() for idx, _ in calls]

    from scmp_kernels_b200 import dist as SD

    def one_call(ai, b_, ci):
        if world > 1:  # this rank's column block, all-gathered into the full output
            return SD.sc_matmul_sharded(ai, b_, M, **ci)
        return sc_matmul(ai, b_, **ci)

    def step(a_list=a_parts, b_=b):
        ys = [one_call(ai, b_, ci) for ai, (_, ci) in zip(a_list, calls)]
        if len(ys) == 1:
            return ys[0]
        y = torch.empty(a.shape[:-1] + (M,), dtype=torch.float32, device=dev)
        for (idx, _), yi in zip(calls, ys):
            y[idx] = yi
        return y

    # rank 0's GPU is sampled from warm-up to the end of the timed steps (the
    # line reports rank 0's clocks); the other GPUs are not polled, since an
    # nvidia-smi query can briefly stall a GPU and the per-call barrier of the
    # sharded path would pass every rank's stall on to all of them
    clk_p, clk_f = clocks_start(local) if rank == 0 else (None, None)
    if clk_p is not None:
        clocks_wait_first_sample(clk_f)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # GEMM-only timing through the library's profiling hook
    L_ = _lib.lib()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps * len(calls))]
    for e0, e1 in ev:  # torch creates the CUDA event on first record
        e0.record()
        e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    t0.record()
    ei = 0
    for _ in range(args.steps):
        ys = []
        for ai, (_, ci) in zip(a_parts, calls):
            L_.scmp_set_profile_events(ev[ei][0]._as_parameter_, ev[ei][1]._as_parameter_)
            ys.append(one_call(ai, b, ci))
            ei += 1
        L_.scmp_set_profile_events(None, None)
        if len(ys) > 1:
            y = torch.empty(a.shape[:-1] + (M,), dtype=torch.float32, device=dev)
            for (idx, _), yi in zip(calls, ys):
                y[idx] = yi
        else:
            y = ys[0]
    t1.record()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    clocks = clocks_stop(clk_p, clk_f)
    ms = t0.elapsed_time(t1) / args.steps
    gemm_ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / args.steps
    if world > 1:
        tt = torch.tensor([ms, gemm_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, gemm_ms = tt.tolist()
    assert _lib.device_error() == 0, "device-side error during the bench"

    ops = 2.0 * BH * N * M * D
    value = ops / (ms * 1e-3) / 1e9

    # end-to-end through the public API from pinned host memory
    e2e = None
    if not args.no_e2e:
        ha = [x.cpu().pin_memory() for x in a_parts]
        hb = b.cpu().pin_memory()
        hs = s.cpu().pin_memory() if s is not None else None
        hy = torch.empty(y.shape, dtype=torch.float32).pin_memory()
        n_e2e = max(1, min(args.steps, 5))
        if world == 1 and len(calls) == 1:
            # the public API on pinned host operands: it streams b to the
            # device and the result back in blocks while it computes
            ci_host = dict(calls[0][1])
            if hs is not None:
                ci_host["smooth_scales"] = hs

            def e2e_step():  # returns the result in pinned host memory
                return sc_matmul(ha[0], hb, **ci_host)
        else:
            def e2e_step():
                da = [x.to(dev, non_blocking=True) for x in ha]
                db = hb.to(dev, non_blocking=True)
                if hs is not None:
                    for _, ci in calls:
                        ci["smooth_scales"] = hs.to(dev, non_blocking=True)
                yy = step(da, db)
                hy.copy_(yy, non_blocking=True)
        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n_e2e):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / n_e2e
        if world > 1:
            tt = torch.tensor([e_ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = tt.item()
        bi = sum(x.numel() * 4 for x in ha) + hb.numel() * 4 + (hs.numel() * 4 if hs is not None else 0)
        e2e = {"value": ops / (e_ms * 1e-3) / 1e9, "unit": "GOPS", "h2d_bytes_per_step": bi,
               "d2h_bytes_per_step": hy.numel() * 4, "ms_per_step": e_ms}

    if rank == 0:
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
            src = "measured"
        except OSError:
            src = "fallback"
        bf16 = peaks.get("bf16_tflops", 1590.0)
        # The SC-GEMM is a GEMM over K = D*L with operands in {-1, 0, 1} (sign x
        # thermometer, sign x stream). SM pairs run it on e2m1 operands
        # (kind::mxf4, dense rate 4x bf16) for streams of 64 positions or more,
        # else on int8 operands (kind::i8, dense rate 2x bf16).
        env = os.environ
        e2m1 = (env.get("SCMP_TC_INT8") != "1" and env.get("SCMP_TC_ATMEM") != "1"
                and env.get("SCMP_TC_SINGLE") != "1" and (L is None or L > 32))
        tc_peak = (4.0 if e2m1 else 2.0) * bf16
        tc_unit = "TOPS (e2m1)" if e2m1 else "TOPS (int8)"
        tc_src = (f"4 x bf16_tflops of {src} peaks (dense e2m1 = 4 x dense bf16)" if e2m1 else
                  f"2 x bf16_tflops of {src} peaks (dense int8 = 2 x dense bf16)")
        Lw = L if L is not None else 149.33
        tensor_ops = 2.0 * BH * N * (M // world if world > 1 else M) * D * Lw
        achieved = tensor_ops / (gemm_ms * 1e-3) / 1e12
        line = {
            "metric": "SC-GEMM equiv GOPS (2*BH*N*M*D/s)", "value": value, "unit": "GOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e2m1xe2m1->f32 (exact integer sums)" if e2m1 else "int8xint8->int32",
            "data": "synthetic (seeded, reference shapes and distributions)",
            "config": {"workload": args.workload, "desc": WORKLOADS[args.workload],
                       "l2": "inputs larger than L2 (b is 180 MB fp32)" if args.workload == "config2" else
                       "per-step operands re-read from HBM",
                       "parallelism": f"b sharded by rows x{world}, NCCL all-gather of outputs" if world > 1
                       else "single GPU"},
            "gpu_launches": launches,
            "gemm_ms_per_step": gemm_ms,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": tc_unit,
                         "frac": achieved / tc_peak,
                         "traffic": (GEMM_TRAFFIC_BYTES.get(args.workload) if shape is None and world == 1
                                     else None),
                         "peak_source": tc_src},
            "clocks": clocks,
            "e2e": e2e,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.workload)
        print(json.dumps(line), flush=True)
    if world > 1:
        SD.release_peer_buffers()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
