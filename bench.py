"""Benchmark of the B200 stochastic-computing matmul (one JSON line on rank 0).

python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config2|config5|config3qk|config3av|config4]
                [--side config5,...|none] [--impl ours|reference]

Metric: equivalent SC-GEMM throughput, 2*BH*N*M*D / t, in GOPS (the
reference's headline), with bit-ops/s = BH*N*M*D*L / t beside it. A step is
one sc_matmul over the workload's resident operands. At N > 1 the weight
operand b is sharded by rows over the ranks and each rank's column block is
stored into every rank's full output by the GEMM's own epilogue (strong
scaling: the job's total work is fixed). `value` is device-timed (CUDA
events, max over ranks); `e2e` times the public API end to end from pinned
host buffers (inputs copied host->device and the result read back every
step; at N > 1 each rank copies in a and its shard of b and reads back its
own column block). At N > 1 the line carries `check`: every rank compares
the first and the last 128 rows of its gathered output with a single-GPU
sc_matmul of those rows against the whole of b, bit for bit, and the run
exits non-zero on a mismatch. `--side` adds the same measurement of other
workloads as nested objects (default: config 5, the north_star's scaling
shape, at every N).

At N = 1 rank 0 also reports: `cpu_baseline`, the C/OpenMP restatement of
the reference's algorithm on a bounded row slice with all host threads;
`reference_gpu`, the reference's own Triton path run on this B200
(baseline/reference_runs.py gpu) with its output compared bit for bit;
`cpu_baseline_interpreter`, the reference's own CPU path (the Triton
interpreter) on configuration 1. `--impl reference` times the C restatement
as the reference arm.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

WORKLOADS = {
    "config2": "per_row bipolar, Llama-7B MLP up-proj: a 4096x4096, b 11008x4096, p=8, L=256",
    "config5": "per_row unipolar + SmoothQuant, Llama-70B MLP: a 8192x8192, b 28672x8192, p=6, L=64",
    "config3qk": "per_head bipolar ViT-B/16 QK: 768 x (197x64) x (197x64), p=8, L=256",
    "config3av": "per_head bipolar ViT-B/16 softmax.V: 768 x (197x197) x (64x197), p=8, L=256",
    "config4": "per_row bipolar chunk_d=64 ViT-B fc2: a 12608x3072, b 768x3072, p=8, L=256/128/64 by row-range tercile",
}

# DRAM bytes (read + write) of one GEMM launch of the full workload on one
# GPU, from a one-pass ncu capture (dram__bytes_read.sum + dram__bytes_write.sum)
GEMM_TRAFFIC_BYTES = {"config2": 314.885376e6 + 200.790272e6, "config5": 3151.572736e6 + 971.502592e6}

# How each workload's inputs stand to the 126 MB L2 between timed steps (no
# flush is issued: the workloads the driver runs have inputs larger than L2)
L2_NOTE = {
    "config2": "inputs larger than L2 (b is 180 MB fp32)",
    "config5": "inputs larger than L2 (a 268 MB, b 940 MB fp32)",
    "config4": "inputs larger than L2 (a is 155 MB fp32)",
    "config3qk": "inputs smaller than L2 (39 MB each, no flush); each step writes a 119 MB result",
    "config3av": "a larger than L2 (119 MB), b 39 MB (no flush); each step writes a 39 MB result",
}

# Dense tensor-core multiply-accumulates per SM and clock on B200, by operand
# type (bf16 4096, int8 8192, e2m1 16384), for the fraction of the nominal
# rate at the sampled SM clock.
MACS_PER_SM_CLK = {"e2m1": 16384, "int8": 8192}
B200_SMS = 148


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="config2", choices=sorted(WORKLOADS))
    ap.add_argument("--side", default="config5",
                    help="comma-separated extra workloads measured the same way, or 'none'")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-runs", action="store_true",
                    help="skip the reference's GPU and interpreter runs at N=1")
    ap.add_argument("--shape", default=None,
                    help="N,M,D override of the config2/config5 recipes (smaller cases for profiling)")
    return ap.parse_args()


def build_workload(name, device, shape=None):
    """(a, b, smooth_scales, kwargs, (BH, N, M, D), L) of a workload."""
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


# ---------------------------------------------------------------------------
# clocks: NVML read in-process (the fields of nvidia-smi's clocks query, read
# only; a sampler subprocess polling the GPU was seen to stall it), with the
# nvidia-smi subprocess as the fallback
# ---------------------------------------------------------------------------

class ClockSampler:
    def __init__(self, cuda_index: int, period_s: float = 0.2):
        self.period, self.samples, self.kind = period_s, [], None
        self._stop, self._thread, self._proc, self._file = threading.Event(), None, None, None
        try:
            import pynvml as P
            import torch
            P.nvmlInit()
            try:
                h = P.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(cuda_index).uuid))
            except Exception:  # noqa: BLE001
                h = P.nvmlDeviceGetHandleByIndex(cuda_index)
            self.P, self.h, self.kind = P, h, "nvml"
            self.max_mhz = float(P.nvmlDeviceGetMaxClockInfo(h, P.NVML_CLOCK_SM))
            self.bits = {"hw_slowdown": P.nvmlClocksEventReasonHwSlowdown,
                         "hw_thermal_slowdown": P.nvmlClocksEventReasonHwThermalSlowdown,
                         "sw_thermal_slowdown": P.nvmlClocksEventReasonSwThermalSlowdown,
                         "sw_power_cap": P.nvmlClocksEventReasonSwPowerCap}
        except Exception:  # noqa: BLE001
            self.kind = "nvidia-smi"
            self.idx = cuda_index

    def _loop(self):
        P, h = self.P, self.h
        while not self._stop.is_set():
            try:
                # SM clock and throttle reasons only: with the board power read
                # in the same loop, the first step's launches were held up
                # (1 run in 40 against 0 in 40 without it, 2 bench runs in 9)
                sm = float(P.nvmlDeviceGetClockInfo(h, P.NVML_CLOCK_SM))
                rs = int(P.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((sm, self.max_mhz, None, [n for n, b in self.bits.items() if rs & b],
                                     time.perf_counter()))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def start(self):
        """Start sampling and return once the first sample is in: the
        sampler's first driver queries then happen before the timed region
        opens. (Started just before the region, they delayed the host's first
        launches in about one run in four while the GPU's queue was empty:
        4-12 ms of idle GPU at the first step.)"""
        self.samples = []
        self._t_open = None
        self._stop.clear()
        if self.kind == "nvml":
            self._thread = threading.Thread(target=self._loop, daemon=True)
            self._thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 2.0:
                time.sleep(0.002)
            return
        import tempfile
        self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False).name
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self._proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={q}",
                                           "--format=csv,noheader,nounits", "-lms", "200"],
                                          stdout=open(self._file, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self._proc = None
        t0 = time.time()  # let the sampler start before the timed region
        while self._proc is not None and time.time() - t0 < 10 and os.path.getsize(self._file) == 0:
            time.sleep(0.05)

    def mark(self):
        """The timed region opens now: samples taken before are dropped (while
        one at least falls inside the region)."""
        self._t_open = time.perf_counter()

    def stop(self):
        if self.kind == "nvml":
            self._stop.set()
            if self._thread is not None:
                self._thread.join(timeout=5)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in open(self._file):
                f = [x.strip() for x in line.split(",")]
                try:
                    self.samples.append((float(f[1]), float(f[2]), float(f[3]),
                                         [n for n, v in zip(names, f[5:9]) if v.lower() == "active"]))
                except (ValueError, IndexError):
                    continue
            os.unlink(self._file)
        if not self.samples:
            return None
        if self.kind == "nvml" and self._t_open is not None:
            inside = [x for x in self.samples if x[4] >= self._t_open]
            if inside:
                self.samples = inside
        mx = self.samples[-1][1]
        sms = [s[0] for s in self.samples]
        load = [s for s in sms if mx and s > 0.5 * mx] or sms
        reasons = sorted({r for s in self.samples for r in s[3]})
        out = {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": reasons,
               "samples": len(sms), "sampler": self.kind}
        power = [s[2] for s in self.samples if s[2] is not None]
        if power:
            out["power_w_max"] = max(power)
        return out


# ---------------------------------------------------------------------------
# baselines on the host cores and the reference's own paths
# ---------------------------------------------------------------------------

def cpu_baseline(workload, max_seconds=20.0):
    """Time the C restatement of the reference's algorithm (test
    infrastructure, used only as this baseline) on a bounded row sample of
    the workload; returns the baseline dict."""
    import numpy as np
    import torch
    from oracle import sc_oracle as O
    from scmp_kernels_b200 import workloads as W
    threads = os.cpu_count() or 1
    try:
        from oracle import c_oracle as CO
        have_c = CO.available()
    except Exception:  # noqa: BLE001
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

    def call(rows):
        sa, sb = np.ascontiguousarray(an[..., :rows, :]), np.ascontiguousarray(bn[..., :rows, :])
        t0 = time.perf_counter()
        if have_c:
            CO.sc_matmul(sa, sb, gran, threads=threads, **q)
        else:
            O.sc_matmul(sa, sb, gran, env={}, **q)
        return time.perf_counter() - t0

    # untimed first call: sequences and tables are built once per key and
    # cached, as the reference's RNG and table caches keep them
    call(8)
    rows = 8
    while True:
        dt = call(rows)
        if dt > max_seconds / 4 or rows >= an.shape[-2]:
            break
        rows = min(an.shape[-2], rows * 2)
    bh = a.shape[0] if a.dim() == 3 else 1
    ops = 2.0 * bh * rows * rows * D
    return {"value": ops / dt / 1e9, "unit": "GOPS", "cores": threads if have_c else 1,
            "kind": "port", "bit_ops_per_s": ops / 2 * L / dt,
            "sample": f"{gran} {workload} slice: {bh}x{rows}x{rows}x{D} (L={L}) in {dt:.2f}s, "
                      f"{'C restatement, OpenMP' if have_c else 'numpy restatement, 1 thread'}"}


def reference_run(mode: str, timeout_s: float, budget_s: float = 60.0):
    """One of baseline/reference_runs.py's measurements in a subprocess."""
    cmd = [sys.executable, os.path.join(REPO, "baseline", "reference_runs.py"), mode, "--budget-s", str(budget_s)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"did not finish within {timeout_s:.0f} s"}
    for line in reversed(r.stdout.strip().splitlines()):
        try:
            return json.loads(line)
        except ValueError:
            continue
    return {"unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout).strip()[-300:]}"}


def run_reference(args, rank, world):
    """--impl reference: the C restatement on the host cores, rank 0 only."""
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


# ---------------------------------------------------------------------------
# one workload, timed
# ---------------------------------------------------------------------------

def measure(name, shape, args, rank, world, dev, sampler=None, check_rows=128):
    import torch
    import torch.distributed as dist
    from scmp_kernels_b200 import _lib, sc_matmul, sc_matmul_levels
    from scmp_kernels_b200 import dist as SD

    a, b_full, s, kw, (BH, N, M, D), L = build_workload(name, dev, shape)
    lo, hi = (0, M)
    b = b_full
    if world > 1:
        lo, hi = SD.shard_bounds(M, world, rank)
        b = b_full[..., lo:hi, :].contiguous()
    kw = dict(kw)
    if s is not None:
        kw["smooth_scales"] = s
    if name == "config4":
        # the caller's mixed precision: row groups of 4 by range tercile, one
        # call with a stream length per row (sc_matmul_levels)
        from scmp_kernels_b200 import workloads as W
        rl, Ls = W.mp_row_level_index(a, 4, (256, 128, 64))
        kw = dict(kw, row_levels=rl, stoc_len_levels=Ls, rng_levels="stoc_len")
    calls = [(None, kw)]
    a_parts = [a if idx is None else a[idx].contiguous() for idx, _ in calls]

    def mm(ai, b_, ci):
        if "row_levels" in ci:
            return sc_matmul_levels(ai, b_, **ci)
        return sc_matmul(ai, b_, **ci)

    def one_call(ai, b_, ci):
        if world > 1:  # this rank's column block, stored into every rank's output
            return SD.sc_matmul_sharded(ai, b_, M, copy=False, **ci)
        return mm(ai, b_, ci)

    def assemble(ys):
        if len(ys) == 1:
            return ys[0]
        y = torch.empty(a.shape[:-1] + (M,), dtype=torch.float32, device=dev)
        for (idx, _), yi in zip(calls, ys):
            y[idx] = yi
        return y

    for _ in range(args.warmup):
        assemble([one_call(ai, b, ci) for ai, (_, ci) in zip(a_parts, calls)])
    torch.cuda.synchronize()

    L_ = _lib.lib()
    nev = args.steps * len(calls)
    mk = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    gev = [(mk(), mk()) for _ in range(nev)]
    qev = [(mk(), mk()) for _ in range(nev)]
    for e0, e1 in gev + qev:  # torch creates the CUDA event on first record
        e0.record()
        e1.record()
    if sampler is not None:  # running (first sample taken) before the region opens
        sampler.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = mk(), mk()
    launches0 = _lib.launch_count()
    if sampler is not None:
        sampler.mark()
    t0.record()
    ei = 0
    for _ in range(args.steps):
        ys = []
        for ai, (_, ci) in zip(a_parts, calls):
            L_.scmp_set_profile_events(gev[ei][0]._as_parameter_, gev[ei][1]._as_parameter_)
            L_.scmp_set_quant_profile_events(qev[ei][0]._as_parameter_, qev[ei][1]._as_parameter_)
            ys.append(one_call(ai, b, ci))
            ei += 1
        L_.scmp_set_profile_events(None, None)
        L_.scmp_set_quant_profile_events(None, None)
        y = assemble(ys)
    t1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler is not None else None
    launches = _lib.launch_count() - launches0
    ms = t0.elapsed_time(t1) / args.steps
    gemm_ms = sum(e0.elapsed_time(e1) for e0, e1 in gev) / args.steps
    quant_ms = sum(e0.elapsed_time(e1) for e0, e1 in qev) / args.steps
    if world > 1:
        tt = torch.tensor([ms, gemm_ms, quant_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, gemm_ms, quant_ms = tt.tolist()
    assert _lib.device_error() == 0, "device-side error during the bench"

    ops = 2.0 * BH * N * M * D
    Lw = L if L is not None else 149.33
    res = {"workload": name, "desc": WORKLOADS[name], "value": ops / (ms * 1e-3) / 1e9, "unit": "GOPS",
           "ms_per_step": ms, "gemm_ms_per_step": gemm_ms, "quant_ms_per_step": quant_ms,
           "bit_ops_per_s": ops / 2 * Lw / (ms * 1e-3), "gpu_launches": launches, "clocks": clocks,
           "_tensor_ops_per_rank": 2.0 * BH * N * (hi - lo) * D * Lw}
    # quantiser: read 4 B per element of a and b, write its 2-byte operand
    # (the row statistics and scales are O(rows))
    res["_quant_bytes"] = 6.0 * BH * (N + (hi - lo)) * D

    # multi-GPU: the gathered output against single-GPU row slices
    if world > 1 and len(calls) == 1 and BH == 1:
        rows = sorted(set(range(min(check_rows, N))) | set(range(max(0, N - check_rows), N)))
        idx = torch.tensor(rows, device=dev)
        ok_t = torch.ones(1, device=dev)
        kw_rows = dict(kw, row_levels=kw["row_levels"][idx]) if "row_levels" in kw else kw
        ref = mm(a[idx].contiguous(), b_full, kw_rows)
        if not torch.equal(y[idx], ref):
            ok_t.zero_()
        dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
        res["check"] = {"bit_exact": bool(ok_t.item() == 1), "rows": len(rows),
                        "how": "every rank's gathered output vs single-GPU sc_matmul of those rows of a "
                               "against the whole of b"}
    del y

    # end to end through the public API from pinned host memory
    if not args.no_e2e:
        ha = [x.cpu().pin_memory() for x in a_parts]
        hb = b.cpu().pin_memory()
        hs = s.cpu().pin_memory() if s is not None else None
        n_e2e = max(1, min(args.steps, 5))
        out_bytes = N * (hi - lo) * 4 * BH
        if len(calls) == 1:
            ci_host = dict(calls[0][1])
            if hs is not None:
                ci_host["smooth_scales"] = hs
            if "row_levels" in ci_host:  # the row levels come from the host too
                ci_host["row_levels"] = ci_host["row_levels"].cpu().pin_memory()
            if world > 1:
                def e2e_step():  # this rank's column block back to host memory, no gather
                    return SD.sc_matmul_sharded(ha[0], hb, M, gather=False, **ci_host)
            else:
                def e2e_step():  # streamed host path; result in pinned host memory
                    return mm(ha[0], hb, ci_host)
        else:
            hy = torch.empty(a.shape[:-1] + ((hi - lo) if world > 1 else M,), dtype=torch.float32).pin_memory()

            def e2e_step():
                da = [x.to(dev, non_blocking=True) for x in ha]
                db = hb.to(dev, non_blocking=True)
                ys = [SD.sc_matmul_sharded(ai, db, M, gather=False, **ci) if world > 1 else sc_matmul(ai, db, **ci)
                      for ai, (_, ci) in zip(da, calls)]
                hy.copy_(assemble(ys), non_blocking=True)
        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = mk(), mk()
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
        if len(calls) == 1 and "row_levels" in ci_host:
            bi += ci_host["row_levels"].numel() * 4
        res["e2e"] = {"value": ops / (e_ms * 1e-3) / 1e9, "unit": "GOPS", "h2d_bytes_per_step": bi,
                      "d2h_bytes_per_step": out_bytes, "ms_per_step": e_ms,
                      "output": ("each rank's column block of the result to its host memory (the result "
                                 "stays sharded by columns)") if world > 1 else "the whole result"}
    del a, b, b_full, a_parts
    torch.cuda.empty_cache()
    return res


def roofline_of(res, args, world, peaks, src, shape):
    """Tensor-core roofline of the GEMM kernel and HBM roofline of the quantiser."""
    bf16 = peaks.get("bf16_tflops", 1590.0)
    hbm = peaks.get("hbm_gbs", 6650.0)
    env = os.environ
    L = {"config5": 64}.get(res["workload"], 256 if res["workload"] != "config4" else None)
    e2m1 = (env.get("SCMP_TC_INT8") != "1" and env.get("SCMP_TC_ATMEM") != "1"
            and env.get("SCMP_TC_SINGLE") != "1" and (L is None or L > 32))
    kind = "e2m1" if e2m1 else "int8"
    tc_peak = (4.0 if e2m1 else 2.0) * bf16
    achieved = res["_tensor_ops_per_rank"] / (res["gemm_ms_per_step"] * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": f"TOPS ({kind})",
            "frac": achieved / tc_peak,
            "traffic": (GEMM_TRAFFIC_BYTES.get(res["workload"]) if shape is None and world == 1 else None),
            "peak_source": f"{'4' if e2m1 else '2'} x bf16_tflops of {src} peaks (dense {kind} = "
                           f"{'4' if e2m1 else '2'} x dense bf16)"}
    clk = res.get("clocks") or {}
    if clk.get("sm_mhz"):
        nominal = B200_SMS * MACS_PER_SM_CLK[kind] * 2 * clk["sm_mhz"] * 1e6 / 1e12
        roof["nominal_at_sampled_clock"] = nominal
        roof["frac_of_nominal_at_sampled_clock"] = achieved / nominal
    q_gbs = res["_quant_bytes"] / (res["quant_ms_per_step"] * 1e-3) / 1e9 if res["quant_ms_per_step"] > 0 else None
    quant = {"bound": "hbm", "achieved": q_gbs, "peak": hbm, "unit": "GB/s",
             "frac": (q_gbs / hbm) if q_gbs else None, "bytes_per_step": res["_quant_bytes"],
             "ms_per_step": res["quant_ms_per_step"],
             "what": "operand preparation per step (row statistics, quantisers, padded row map): "
                     "4 B read + 2 B written per element of a and of this rank's b"}
    return roof, quant


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from scmp_kernels_b200 import dist as SD

    shape = tuple(int(x) for x in args.shape.split(",")) if args.shape else None
    # rank 0's GPU is sampled during each timed region (the line reports rank
    # 0's clocks); the other GPUs are not polled
    sampler = ClockSampler(local) if rank == 0 else None
    head = measure(args.workload, shape, args, rank, world, dev, sampler)
    sides = []
    if args.side and args.side != "none" and shape is None:
        for w in args.side.split(","):
            if w and w != args.workload:
                sides.append(measure(w, None, args, rank, world, dev, sampler))
    failed = [r["workload"] for r in [head] + sides if r.get("check") and not r["check"]["bit_exact"]]

    if rank == 0:
        peaks, src = {}, "fallback"
        try:
            peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
            src = "measured"
        except OSError:
            pass
        roof, quant = roofline_of(head, args, world, peaks, src, shape)
        e2m1 = roof["unit"].endswith("(e2m1)")
        line = {
            "metric": "SC-GEMM equiv GOPS (2*BH*N*M*D/s)", "value": head["value"], "unit": "GOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e2m1xe2m1->f32 (exact integer sums)" if e2m1 else "int8xint8->int32",
            "data": "synthetic (seeded, reference shapes and distributions)",
            "config": {"workload": args.workload, "desc": WORKLOADS[args.workload],
                       "l2": L2_NOTE[args.workload],
                       "parallelism": (f"b sharded by rows x{world}, each rank's block stored into every "
                                       f"rank's output by the GEMM epilogue (NVLink)") if world > 1
                       else "single GPU"},
            "gpu_launches": head["gpu_launches"],
            "gemm_ms_per_step": head["gemm_ms_per_step"],
            "bit_ops_per_s": head["bit_ops_per_s"],
            "roofline": roof,
            "quant_roofline": quant,
            "clocks": head["clocks"],
            "e2e": head.get("e2e"),
        }
        if "check" in head:
            line["check"] = head["check"]
        for r in sides:
            r_roof, r_quant = roofline_of(r, args, world, peaks, src, None)
            line[r["workload"]] = {k: v for k, v in r.items() if not k.startswith("_")}
            line[r["workload"]]["roofline"] = r_roof
            line[r["workload"]]["quant_roofline"] = r_quant
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.workload)
        if world == 1 and not args.no_reference_runs and shape is None:
            line["reference_gpu"] = reference_run("gpu", timeout_s=300, budget_s=60)
            line["cpu_baseline_interpreter"] = reference_run("interp", timeout_s=300)
        print(json.dumps(line), flush=True)
    if world > 1:
        SD.release_peer_buffers()
        dist.barrier()
        dist.destroy_process_group()
    if failed:
        sys.stderr.write(f"bench: multi-GPU output check failed for {failed}\n")
        sys.exit(3)


if __name__ == "__main__":
    main()
