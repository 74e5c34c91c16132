"""The reference's own code paths, timed beside this library's.

Runs the unmodified reference package ``scmp_kernels`` (swalther06/scmp_kernels)
installed in ``baseline/_ref`` (``pip install --no-index --no-build-isolation
--no-deps --target baseline/_ref <reference checkout>``). Two modes, each
printing one JSON line:

gpu     The reference's ``sc_matmul`` on the B200 through its stock path: its
        Triton table kernels (``build_cum_indicator_kernel``,
        ``compute_k_table_kernel``), its torch quantisers and its
        ``enable_matmul_tiled_kernel`` (sc/kernels.py:102-169, 176-252,
        798-868, 1573-1707), JIT-compiled by the installed Triton, on the
        config-2 workload (per_row bipolar, a 4096x4096 with outlier channels,
        b 11008x4096, p = 8, L = 256). The first call (compile and table build)
        is untimed. When a full call would take longer than the budget, the
        first rows of a are timed instead (the reference's grid is over output
        tiles, so its time is proportional to the rows) and the line says so.
        The reference's output is then compared bit for bit with this
        library's on the same rows.

interp  The reference's CPU path: ``sc_matmul`` under ``TRITON_INTERPRET=1``
        (every Triton op evaluated by numpy) with two host shims that leave
        the arithmetic alone (``Tensor.cuda`` is the identity, and
        ``libdevice.nearbyint``, an extern call the interpreter cannot run, is
        ``numpy.rint``: the same round-half-to-even), on config 1 (per_tensor
        bipolar, a 64x256, b 32x256 from seed 0, the LFSR default config with
        taps [7, 2, 1, 0] and seed 125). The cold call builds the tables with
        the reference's two table kernels launched on row slices by a pool of
        processes (each program of those kernels touches only its own row);
        the warm call runs in one process (the interpreter is single-threaded).

Usage: python baseline/reference_runs.py gpu|interp [--budget-s S]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")


def _unavailable(why: str) -> None:
    print(json.dumps({"unavailable": why}), flush=True)


def run_gpu(budget_s: float) -> None:
    import torch
    if not torch.cuda.is_available():
        return _unavailable("no CUDA device")
    try:
        import triton
    except Exception as e:  # noqa: BLE001
        return _unavailable(f"triton not importable: {e}")
    if not os.path.isdir(os.path.join(REF, "scmp_kernels")):
        return _unavailable("reference package not installed in baseline/_ref")
    sys.path.insert(0, REF)
    sys.path.insert(1, REPO)
    from scmp_kernels import sc_matmul as ref_sc_matmul
    from scmp_kernels_b200 import sc_matmul, workloads

    dev = torch.device("cuda", 0)
    a, b = workloads.config2(dev)
    n, m, d = a.shape[0], b.shape[0], a.shape[1]
    kw = dict(mode="bipolar", sc_prec=8)

    def timed(x, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            y = ref_sc_matmul(x, b, "per_row", **kw)
        e1.record()
        torch.cuda.synchronize()
        return y, e0.elapsed_time(e1) / reps

    probe_rows = 256
    t0 = time.perf_counter()
    ref_sc_matmul(a[:probe_rows].contiguous(), b, "per_row", **kw)  # compile + tables
    torch.cuda.synchronize()
    cold_s = time.perf_counter() - t0
    xa = a[:probe_rows].contiguous()
    _, probe_ms = timed(xa, 1)
    est_full_s = probe_ms * 1e-3 * n / probe_rows
    rows = probe_rows
    if 2 * est_full_s <= budget_s:
        rows = n
    elif 2 * est_full_s * 1024 / n <= budget_s:
        rows = 1024
    xa = a[:rows].contiguous()
    reps = 2 if rows < n or 3 * est_full_s <= budget_s else 1
    y_ref, ms = timed(xa, reps)
    y_ours = sc_matmul(xa, b, "per_row", **kw)
    torch.cuda.synchronize()
    mism = int((y_ref != y_ours).sum().item())
    ops = 2.0 * rows * m * d
    line = {
        "value": ops / (ms * 1e-3) / 1e9, "unit": "GOPS", "ms_per_call": ms, "rows_of_a": rows,
        "workload": "config2" if rows == n else f"config2, first {rows} of {n} rows of a",
        "calls_timed": reps, "cold_first_call_s": cold_s,
        "triton": triton.__version__, "torch": torch.__version__,
        "kernel": "enable_matmul_tiled_kernel (reference default table path)",
        "end_to_end": {"bit_exact_vs_ours": mism == 0, "mismatches": mism, "elements_compared": rows * m},
    }
    del y_ref, y_ours
    line["gemm_kernel"] = _compare_gemm_kernels(xa, b)
    line["row_scales"] = _compare_row_scales(xa, b)
    print(json.dumps(line), flush=True)


def _compare_gemm_kernels(xa, b):
    """The reference's GEMM kernel (enable_matmul_triton) and this library's
    (scmp_enable_matmul) on the same quantised operands: the reference's own
    quantisation of a and b on this GPU."""
    import torch
    import scmp_kernels.sc.kernels as RK
    from scmp_kernels.quant.grouped import _grouped_symmetric_quant as ref_gq
    from scmp_kernels.sc.config_helpers import make_sobol_simple_config as ref_cfg
    from scmp_kernels_b200.sc import kernels as K
    from scmp_kernels_b200.sc.config_helpers import make_sobol_simple_config
    n, d = xa.shape
    m = b.shape[0]
    q, G, L = 127, 256, 256
    _, a_int, sign_a = ref_gq(xa, 1, q)
    _, b_int, sign_b = ref_gq(b, 1, q)
    ba = (a_int.abs() * G / q).round().short()
    bb = (b_int.abs() * G / q).round().short()
    cfg = ref_cfg(d, d, 8)
    ra, rb = RK._get_cached_sequences(cfg, 8, xa.device)
    cum, kt = RK._get_cached_enable_tables(cfg, 8, xa.device, ra, rb, L, rng_levels=G)
    raw_ref = RK.enable_matmul_triton(cum, kt, ba, bb, sign_a, sign_b, n, m, d, L, float(q * q), True)
    del cum
    t = K._get_cached_enable_tables(make_sobol_simple_config(d, d, 8), 8, xa.device, L, G)
    raw_ours = K.enable_matmul(t, ba, bb, sign_a, sign_b, n, m, d, L, float(q * q), True)
    torch.cuda.synchronize()
    mism = int((raw_ref != raw_ours).sum().item())
    return {"bit_exact": mism == 0, "mismatches": mism, "elements_compared": n * m,
            "what": "fl32(S * q_max^2 / L) of enable_matmul_triton vs scmp_enable_matmul on the reference's "
                    "own boundaries and signs of a and b"}


def _compare_row_scales(xa, b):
    """The per-row scale absmax / q_max of the reference's grouped quantiser,
    as torch evaluates it on this GPU and on the CPU (which the interpreter
    runs, and which the fixtures and this library follow)."""
    import torch
    from scmp_kernels.quant.grouped import _grouped_symmetric_quant as ref_gq
    out = {}
    for name, x in (("a", xa), ("b", b)):
        s_gpu, i_gpu, _ = ref_gq(x, 1, 127)
        s_cpu, i_cpu, _ = ref_gq(x.cpu(), 1, 127)
        amax = x.abs().amax(dim=1).clamp(min=1e-5).cpu()
        recip = amax * torch.tensor(1.0 / 127, dtype=torch.float32)
        out[name] = {"rows": int(x.shape[0]),
                     "gpu_ne_cpu": int((s_gpu.cpu() != s_cpu).sum()),
                     "cpu_eq_divide": bool(torch.equal(s_cpu, amax / 127)),
                     "gpu_eq_times_reciprocal": bool(torch.equal(s_gpu.cpu(), recip)),
                     "quantised_values_ne": int((i_gpu.cpu() != i_cpu).sum())}
    return out


_ORIG = {}


def _interp_worker(job):
    import numpy as np
    import torch
    kind, rows, stoc_len, V = job
    rng = torch.from_numpy(rows)
    dd = rows.shape[0]
    shape = (dd, stoc_len + 1, V) if kind == "cum" else (dd, V)
    out = torch.zeros(*shape, dtype=torch.int16)
    _ORIG[kind][(dd,)](rng, out, dd, stoc_len, V)
    return np.ascontiguousarray(out.numpy())


class _RowSplit:
    """Launches one of the reference's row-independent table kernels on row
    slices in a process pool and stitches the rows together."""

    def __init__(self, kind, pool, nproc):
        self.kind, self.pool, self.nproc = kind, pool, nproc

    def __getitem__(self, grid):
        import numpy as np
        import torch

        def launch(rng, out, D, stoc_len, V):
            D = int(D)
            rows = rng[:D].contiguous().numpy().astype(np.int32)
            bounds = np.linspace(0, D, 4 * self.nproc + 1).astype(int)
            jobs = [(self.kind, rows[bounds[i]:bounds[i + 1]], int(stoc_len), int(V))
                    for i in range(len(bounds) - 1) if bounds[i + 1] > bounds[i]]
            parts = self.pool.map(_interp_worker, jobs)
            out[:D].copy_(torch.from_numpy(np.concatenate(parts, axis=0)))
        return launch


def run_interp(budget_s: float) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    import multiprocessing as mp

    import numpy as np
    import torch
    if not os.path.isdir(os.path.join(REF, "scmp_kernels")):
        return _unavailable("reference package not installed in baseline/_ref")
    sys.path.insert(0, REF)
    torch.Tensor.cuda = lambda self, *a, **k: self
    import triton.language as tl
    from triton.runtime.interpreter import TensorHandle

    class _LibdeviceShim:
        @staticmethod
        def nearbyint(x, _semantic=None, **kw):
            return tl.core.tensor(TensorHandle(np.rint(x.handle.data), x.handle.dtype.scalar), x.type)

    import scmp_kernels.quant.fused as F
    import scmp_kernels.sc.kernels as K
    from scmp_kernels import sc_matmul
    from scmp_kernels.sc import clear_rng_cache
    from scmp_kernels.sc.config_helpers import make_default_config
    F.libdevice = _LibdeviceShim
    K.libdevice = _LibdeviceShim

    nproc = os.cpu_count() or 1
    _ORIG["cum"], _ORIG["ktab"] = K.build_cum_indicator_kernel, K.compute_k_table_kernel
    # the pool forks (with the kernels above) before this process touches any device
    pool = mp.get_context("fork").Pool(nproc)

    g = torch.Generator().manual_seed(0)
    a = torch.randn(64, 256, generator=g)
    b = torch.randn(32, 256, generator=g)
    cfg = make_default_config(256, 256, 8, taps=[7, 2, 1, 0], seed=125)
    clear_rng_cache()
    K.build_cum_indicator_kernel = _RowSplit("cum", pool, nproc)
    K.compute_k_table_kernel = _RowSplit("ktab", pool, nproc)
    t0 = time.perf_counter()
    sc_matmul(a, b, "per_tensor", mode="bipolar", sc_prec=8, config=cfg)
    cold = time.perf_counter() - t0
    K.build_cum_indicator_kernel, K.compute_k_table_kernel = _ORIG["cum"], _ORIG["ktab"]
    pool.close()
    pool.join()
    t0 = time.perf_counter()
    y = sc_matmul(a, b, "per_tensor", mode="bipolar", sc_prec=8, config=cfg)
    warm = time.perf_counter() - t0
    n, m, d, L = 64, 32, 256, 256
    print(json.dumps({
        "value": 2.0 * n * m * d / warm / 1e9, "unit": "GOPS", "warm_s": warm, "cold_s": cold,
        "bit_ops_per_s": n * m * d * L / warm, "cores_warm": 1, "cores_cold_table_build": nproc,
        "nproc": nproc, "workload": "config1 (per_tensor bipolar 64x256 . 32x256, p=8, L=256, LFSR config)",
        "checksum": float(y.double().sum()),
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["gpu", "interp"])
    ap.add_argument("--budget-s", type=float, default=60.0)
    args = ap.parse_args()
    try:
        (run_gpu if args.mode == "gpu" else run_interp)(args.budget_s)
    except Exception as e:  # noqa: BLE001
        _unavailable(f"{type(e).__name__}: {e}"[:300])


if __name__ == "__main__":
    main()
