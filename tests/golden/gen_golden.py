"""Generate the golden fixtures in this directory by running the reference.

The reference ``scmp_kernels`` is a Python + Triton package. Its own
``sc_matmul`` is executed on the CPU under ``TRITON_INTERPRET=1`` (the
interpreter computes every Triton op with numpy IEEE float32 arithmetic), with
two host-side shims that leave the algorithm untouched:

* ``torch.Tensor.cuda`` becomes the identity, so the ``.cuda()`` moves in the
  reference's path orchestrators keep the tensors on the CPU;
* ``libdevice.nearbyint`` (an extern call the interpreter cannot execute) is
  replaced by ``numpy.rint``, which is the same round-half-to-even.

The reference's two table-building kernels (``build_cum_indicator_kernel`` and
``compute_k_table_kernel``) touch only row ``d`` of their operands in program
``d``; the interpreter runs programs one after another, so for large ``D`` this
script launches the unmodified kernels on row slices in a process pool and
stitches the rows back together. The GEMM, quantisation and epilogue run as the
reference launches them.

Usage:  python tests/golden/gen_golden.py --reference <path to scmp_kernels checkout> [case ...]

Each case writes ``<case>.npz`` holding the inputs, the call parameters (JSON)
and the reference output; ``rng_golden.npz`` holds RNG sequences, prepared
prefixes and tables from the reference's own functions.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import sys
import time

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

_POOL = None
_ORIG = {}
K = F = None


def _install_reference(path: str):
    global K, F
    sys.path.insert(0, path)
    torch.Tensor.cuda = lambda self, *a, **k: self
    import triton.language as tl
    from triton.runtime.interpreter import TensorHandle

    class _LibdeviceShim:
        @staticmethod
        def nearbyint(x, _semantic=None, **kw):
            return tl.core.tensor(
                TensorHandle(np.rint(x.handle.data), x.handle.dtype.scalar), x.type)

    import scmp_kernels.quant.fused as F_
    import scmp_kernels.sc.kernels as K_
    F_.libdevice = _LibdeviceShim
    K_.libdevice = _LibdeviceShim
    K, F = K_, F_
    _ORIG["cum"] = K.build_cum_indicator_kernel
    _ORIG["ktab"] = K.compute_k_table_kernel
    K.build_cum_indicator_kernel = _RowSplit("cum")
    K.compute_k_table_kernel = _RowSplit("ktab")


def _worker(job):
    kind, rows, stoc_len, V = job
    rng = torch.from_numpy(rows)
    d = rows.shape[0]
    if kind == "cum":
        out = torch.zeros(d, stoc_len + 1, V, dtype=torch.int16)
    else:
        out = torch.zeros(d, V, dtype=torch.int16)
    _ORIG[kind][(d,)](rng, out, d, stoc_len, V)
    return out.numpy()


class _RowSplit:
    """Launch the reference's row-independent table kernel on row slices."""

    def __init__(self, kind):
        self.kind = kind

    def __getitem__(self, grid):
        def launch(rng, out, D, stoc_len, V):
            D = int(D)
            rows = rng[:D].contiguous().numpy().astype(np.int32)
            if D < 64 or _POOL is None:
                _ORIG[self.kind][(D,)](rng, out, D, stoc_len, V)
                return
            n = 8 * 4
            bounds = np.linspace(0, D, n + 1).astype(int)
            jobs = [(self.kind, rows[bounds[i]:bounds[i + 1]], stoc_len, V)
                    for i in range(n) if bounds[i + 1] > bounds[i]]
            parts = _POOL.map(_worker, jobs)
            out[:D].copy_(torch.from_numpy(np.concatenate(parts, axis=0)))
        return launch


# --------------------------------------------------------------------------
# cases
# --------------------------------------------------------------------------

def _save(name, out, a, b, params, extra=None):
    d = dict(a=np.asarray(a, dtype=np.float32), b=np.asarray(b, dtype=np.float32),
             out=np.asarray(out, dtype=np.float32),
             params=np.array(json.dumps(params, sort_keys=True)))
    if extra:
        for k, v in extra.items():
            d[k] = np.asarray(v)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **d)


def _run(name, a, b, params, env=None, smooth=None, extra=None):
    from scmp_kernels import sc_matmul
    from scmp_kernels.sc import clear_rng_cache
    env = env or {}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    clear_rng_cache()
    t0 = time.time()
    kw = {k: v for k, v in params.items() if k not in ("granularity", "config_name")}
    if smooth is not None:
        kw["smooth_scales"] = smooth
    y = sc_matmul(a, b, params["granularity"], **kw)
    dt = time.time() - t0
    clear_rng_cache()
    for k, v in old.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v
    p = dict(params)
    p["env"] = env
    ex = dict(extra or {})
    if smooth is not None:
        ex["smooth_scales"] = smooth.numpy()
    _save(name, y.numpy(), a.numpy(), b.numpy(), p, ex)
    print(f"[{name}] out {tuple(y.shape)} in {dt:.1f}s", flush=True)


def _rows(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randperm(n, generator=g)[:k]
    idx[0] = 0
    idx[-1] = n - 1
    return torch.sort(idx).values


def case_cfg1(names):
    from scmp_kernels_b200 import workloads as W
    from scmp_kernels.sc.config_helpers import make_default_config
    a, b = W.config1()
    cfg = make_default_config(256, 256, 8, taps=[7, 2, 1, 0], seed=125)
    if "cfg1_lfsr" in names:
        _run("cfg1_lfsr", a, b, dict(granularity="per_tensor", mode="bipolar", sc_prec=8,
                                     stoc_len=256, config=cfg))
    if "cfg1_sobol" in names:
        _run("cfg1_sobol", a, b, dict(granularity="per_tensor", mode="bipolar", sc_prec=8))
    if "cfg1_unipolar" in names:
        _run("cfg1_unipolar", a, b, dict(granularity="per_tensor", mode="unipolar", sc_prec=8))


def case_cfg2(names):
    from scmp_kernels_b200 import workloads as W
    a, b = W.config2()
    ia, ib = _rows(a.shape[0], 16, 21), _rows(b.shape[0], 16, 22)
    _run("cfg2_slice", a[ia].contiguous(), b[ib].contiguous(),
         dict(granularity="per_row", mode="bipolar", sc_prec=8, stoc_len=256),
         extra=dict(rows_a=ia.numpy(), rows_b=ib.numpy()))


def case_cfg3(names):
    from scmp_kernels_b200 import workloads as W
    q, k, probs, v_t = W.config3()
    heads = torch.tensor([0, 383, 767])
    if "cfg3_qk" in names:
        _run("cfg3_qk", q[heads].contiguous(), k[heads].contiguous(),
             dict(granularity="per_head", mode="bipolar", sc_prec=8),
             extra=dict(heads=heads.numpy()))
    if "cfg3_av" in names:
        _run("cfg3_av", probs[heads].contiguous(), v_t[heads].contiguous(),
             dict(granularity="per_head", mode="bipolar", sc_prec=8),
             extra=dict(heads=heads.numpy()))


def case_cfg4(names):
    from scmp_kernels_b200 import workloads as W
    a, b = W.config4()
    lv = W.mp_row_levels(a, 4, (256, 128, 64))
    ib = _rows(b.shape[0], 16, 42)
    for L, rows in lv.items():
        g = torch.Generator().manual_seed(L)
        pick = rows[torch.randperm(rows.numel(), generator=g)[:12]]
        pick = torch.sort(pick).values
        nm = f"cfg4_L{L}"
        if nm in names:
            _run(nm, a[pick].contiguous(), b[ib].contiguous(),
                 dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=64,
                      group_a=4, group_b=4, stoc_len=L, rng_levels=L),
                 extra=dict(rows_a=pick.numpy(), rows_b=ib.numpy()))
        nm2 = f"cfg4_L{L}_grid256"
        if L == 128 and nm2 in names:
            _run(nm2, a[pick].contiguous(), b[ib].contiguous(),
                 dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=64,
                      group_a=4, group_b=4, stoc_len=L),
                 extra=dict(rows_a=pick.numpy(), rows_b=ib.numpy()))


def case_cfg5(names):
    from scmp_kernels_b200 import workloads as W
    from scmp_kernels.quant.smoothquant import accumulate_act_scales, compute_smooth_scales
    a, b, _ = W.config5(with_scales=False)
    s = compute_smooth_scales(accumulate_act_scales(a), b, alpha=0.5)
    ia, ib = _rows(a.shape[0], 16, 51), _rows(b.shape[0], 16, 52)
    _run("cfg5_slice", a[ia].contiguous(), b[ib].contiguous(),
         dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=64),
         smooth=s, extra=dict(rows_a=ia.numpy(), rows_b=ib.numpy()))


def case_edges(names):
    from scmp_kernels.sc.config_helpers import (
        make_default_config, make_independent_config, make_per_element_scramble_config)
    import random

    def rnd(*shape, seed, scale=1.0):
        g = torch.Generator().manual_seed(seed)
        return torch.randn(*shape, generator=g) * scale

    E = {}
    E["e_rowgroup_bip"] = (rnd(10, 40, seed=101), rnd(12, 40, seed=102),
                           dict(granularity="per_row", mode="bipolar", sc_prec=8, group_a=3, group_b=5))
    E["e_rowgroup_uni"] = (rnd(10, 40, seed=103), rnd(12, 40, seed=104),
                           dict(granularity="per_row", mode="unipolar", sc_prec=8, group_a=3, group_b=1))
    E["e_row_uni_pertensor"] = (rnd(9, 33, seed=105), rnd(7, 33, seed=106),
                                dict(granularity="per_row", mode="unipolar", sc_prec=6, group_a=9, group_b=100))
    E["e_row3d_bip"] = (rnd(3, 6, 40, seed=107), rnd(3, 5, 40, seed=108),
                        dict(granularity="per_row", mode="bipolar", sc_prec=8))
    E["e_row3d_bip_gt"] = (rnd(2, 6, 24, seed=109), rnd(2, 5, 24, seed=110),
                           dict(granularity="per_row", mode="bipolar", sc_prec=8, group_a=6, group_b=99))
    E["e_row3d_uni"] = (rnd(2, 6, 24, seed=111), rnd(2, 5, 24, seed=112),
                        dict(granularity="per_row", mode="unipolar", sc_prec=8, group_a=2))
    E["e_tensor_uni_small"] = (rnd(7, 29, seed=113), rnd(6, 29, seed=114),
                               dict(granularity="per_tensor", mode="unipolar", sc_prec=6))
    E["e_halve"] = (rnd(8, 48, seed=115), rnd(9, 48, seed=116),
                    dict(granularity="per_row", mode="bipolar", sc_prec=8, halve_bipolar_stoc_len=True))
    E["e_prefix64"] = (rnd(8, 48, seed=117), rnd(9, 48, seed=118),
                       dict(granularity="per_row", mode="bipolar", sc_prec=8, stoc_len=64))
    E["e_rescale64"] = (rnd(8, 48, seed=119), rnd(9, 48, seed=120),
                        dict(granularity="per_row", mode="bipolar", sc_prec=8, stoc_len=64, rng_levels=64))
    E["e_rescale_long"] = (rnd(5, 20, seed=121), rnd(6, 20, seed=122),
                           dict(granularity="per_row", mode="bipolar", sc_prec=6, stoc_len=40, rng_levels=100))
    E["e_p4"] = (rnd(6, 30, seed=123), rnd(7, 30, seed=124),
                 dict(granularity="per_row", mode="bipolar", sc_prec=4))
    E["e_p6_uni_prefix"] = (rnd(6, 30, seed=125), rnd(7, 30, seed=126),
                            dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=24))
    E["e_chunk_rem"] = (rnd(6, 100, seed=127), rnd(5, 100, seed=128),
                        dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=32))
    E["e_chunk_ge_d"] = (rnd(6, 30, seed=129), rnd(5, 30, seed=130),
                         dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=32, group_a=2))
    E["e_chunk_short"] = (rnd(6, 70, seed=131), rnd(5, 70, seed=132),
                          dict(granularity="per_row", mode="bipolar", sc_prec=8, chunk_d=24,
                               stoc_len=16, rng_levels=16))
    E["e_zeros"] = (torch.zeros(4, 20), rnd(5, 20, seed=133),
                    dict(granularity="per_row", mode="bipolar", sc_prec=8))
    E["e_zeros_uni"] = (torch.zeros(4, 20), rnd(5, 20, seed=134),
                        dict(granularity="per_row", mode="unipolar", sc_prec=8))
    E["e_tiny"] = (rnd(1, 1, seed=135), rnd(1, 1, seed=136),
                   dict(granularity="per_row", mode="bipolar", sc_prec=8))
    E["e_head_small"] = (rnd(2, 5, 9, seed=137), rnd(2, 7, 9, seed=138),
                         dict(granularity="per_head", mode="bipolar", sc_prec=8))
    E["e_head_prefix"] = (rnd(2, 5, 9, seed=139), rnd(2, 7, 9, seed=140),
                          dict(granularity="per_head", mode="bipolar", sc_prec=6, stoc_len=32, rng_levels=48))
    E["e_tensor_bip_3d"] = None  # per-batch CUDA streams in the reference: not runnable on the CPU
    cfg_ind = make_independent_config(30, 30, 6, q_taps=[5, 0], k_taps=[5, 4, 3, 0],
                                      q_seed=7, k_seed=33)
    E["e_lfsr_indep"] = (rnd(6, 30, seed=141), rnd(7, 30, seed=142),
                         dict(granularity="per_row", mode="bipolar", sc_prec=6, config=cfg_ind))
    random.seed(1234)
    cfg_pe = make_per_element_scramble_config(24, 24, 8, taps=[7, 2, 1, 0], seed=99)
    E["e_lfsr_perelem"] = (rnd(5, 24, seed=143), rnd(6, 24, seed=144),
                           dict(granularity="per_row", mode="bipolar", sc_prec=8, config=cfg_pe))
    E["e_lfsr_perelem_prefix"] = (rnd(5, 24, seed=145), rnd(6, 24, seed=146),
                                  dict(granularity="per_row", mode="unipolar", sc_prec=8, config=cfg_pe,
                                       stoc_len=100))
    cfg_tr = {"rng_pool": [{"type": "true_random", "seed": 7}, {"type": "true_random", "seed": 8}],
              "sng": {"q": [{"rng_id": 0, "scramble": None}] * 16,
                      "k": [{"rng_id": 1, "scramble": [1, 0, 3, 2, 5, 4, 7, 6]}] * 16}}
    E["e_truerandom"] = (rnd(5, 16, seed=147), rnd(4, 16, seed=148),
                         dict(granularity="per_row", mode="bipolar", sc_prec=8, config=cfg_tr))
    cfg_def6 = make_default_config(40, 40, 6, taps=[5, 0], seed=21)
    E["e_tensor_lfsr6"] = (rnd(6, 40, seed=149), rnd(5, 40, seed=150),
                           dict(granularity="per_tensor", mode="bipolar", sc_prec=6, config=cfg_def6))
    for nm, v in E.items():
        if v is None or nm not in names:
            continue
        a, b, p = v
        _run(nm, a, b, p)

    env_cases = {
        "e_owen_counter": ({"SC_OWEN_MODE": "counter"}, 151),
        "e_owen_off": ({"SC_OWEN_MODE": "off"}, 153),
        "e_owen_disable": ({"SC_DISABLE_OWEN": "1"}, 155),
        "e_rescale_noscramble": ({"SC_SCRAMBLE_RESCALE": "0"}, 157),
    }
    for nm, (env, sd) in env_cases.items():
        if nm not in names:
            continue
        p = dict(granularity="per_row", mode="bipolar", sc_prec=8, stoc_len=64)
        if nm == "e_rescale_noscramble":
            p["rng_levels"] = 64
        _run(nm, rnd(8, 48, seed=sd), rnd(9, 48, seed=sd + 1), p, env=env)

    if "e_smooth_row" in names:
        a = rnd(16, 64, seed=160, scale=0.5)
        a[:, 7] *= 30.0
        b = rnd(16, 64, seed=161, scale=0.5)
        from scmp_kernels.quant.smoothquant import accumulate_act_scales, compute_smooth_scales
        s = compute_smooth_scales(accumulate_act_scales(a), b, alpha=0.5)
        _run("e_smooth_row", a, b, dict(granularity="per_row", mode="bipolar", sc_prec=8), smooth=s)
    if "e_smooth_head" in names:
        a = rnd(2, 6, 16, seed=162)
        b = rnd(2, 5, 16, seed=163)
        s = torch.rand(16, generator=torch.Generator().manual_seed(164)) + 0.5
        _run("e_smooth_head", a, b, dict(granularity="per_head", mode="bipolar", sc_prec=8), smooth=s)


def case_configs(names):
    """The Sobol config builders of config_helpers.py:610-763 (antithetic,
    alternative K seed, custom seeds with scrambles, DSE random seeds). The
    reference's make_sobol_dse_config cannot be imported (its ``from rng import
    Sobol`` fails), so that fixture's config comes from this package's builder
    under a fixed ``random`` seed; the reference's sc_matmul consumes it."""
    import random
    from scmp_kernels.sc.config_helpers import (
        make_sobol_altseed_config, make_sobol_antithetic_config, make_sobol_custom_seed_config)
    from scmp_kernels_b200.sc.config_helpers import make_sobol_dse_config

    def rnd(*shape, seed):
        return torch.randn(*shape, generator=torch.Generator().manual_seed(seed))

    C = {}
    C["e_cfg_antithetic"] = (rnd(6, 40, seed=201), rnd(7, 40, seed=202),
                             dict(granularity="per_row", mode="bipolar", sc_prec=8,
                                  config=make_sobol_antithetic_config(40, 40, 8)))
    C["e_cfg_altseed8"] = (rnd(6, 40, seed=203), rnd(7, 40, seed=204),
                           dict(granularity="per_row", mode="bipolar", sc_prec=8,
                                config=make_sobol_altseed_config(40, 40, 8)))
    C["e_cfg_altseed6_prefix"] = (rnd(6, 36, seed=205), rnd(7, 36, seed=206),
                                  dict(granularity="per_row", mode="unipolar", sc_prec=6, stoc_len=40,
                                       config=make_sobol_altseed_config(36, 36, 6)))
    random.seed(77)
    C["e_cfg_custom_seed"] = (rnd(5, 32, seed=207), rnd(6, 32, seed=208),
                              dict(granularity="per_row", mode="bipolar", sc_prec=8,
                                   config=make_sobol_custom_seed_config(
                                       32, 32, 8, q_seed=[1, 1, 3, 5, 15, 17, 51, 85],
                                       k_seed=[1, 3, 7, 1, 9, 33, 41, 255], use_scrambling=True)))
    random.seed(2024)
    C["e_cfg_dse"] = (rnd(5, 32, seed=209), rnd(6, 32, seed=210),
                      dict(granularity="per_tensor", mode="bipolar", sc_prec=8,
                           config=make_sobol_dse_config(32, 32, 8)))
    for nm, (a, b, p) in C.items():
        if nm in names:
            _run(nm, a, b, p)


def case_rng(names):
    """RNG sequences, prepared prefixes and tables from the reference's own functions."""
    from scmp_kernels.sc.rng import Sobol, LFSR
    from scmp_kernels.sc.sng import RNGPool, SNGBank
    from scmp_kernels.sc.lfsr_taps import search_taps
    from scmp_kernels.sc.config_helpers import make_default_config, make_sobol_simple_config
    out = {}
    for p in (4, 6, 8):
        out[f"sobol_q_p{p}"] = Sobol(p, seed_type="q").simulate()
        out[f"sobol_k_p{p}"] = Sobol(p, seed_type="k").simulate()
    out["lfsr_p8_s125"] = LFSR(125, 8, [7, 2, 1, 0]).simulate()
    out["lfsr_p6_s21"] = LFSR(21, 6, [5, 0]).simulate()
    for p in (4, 6, 8):
        out[f"taps_p{p}"] = np.array(search_taps(p, verbose=False)[0])
    cfg = make_default_config(5, 5, 8, taps=[7, 2, 1, 0], seed=125)
    pool = RNGPool(cfg["rng_pool"], 8)
    out["bank_default_q"] = SNGBank(pool, cfg["sng"]["q"]).get_all_sequences(256)
    out["bank_default_k"] = SNGBank(pool, cfg["sng"]["k"]).get_all_sequences(256)
    # prepared prefixes (prefix / Owen / rescale) on a 6-row Sobol-K bank at p=8
    cfg2 = make_sobol_simple_config(6, 6, 8)
    pool2 = RNGPool(cfg2["rng_pool"], 8)
    rb = torch.tensor(SNGBank(pool2, cfg2["sng"]["k"]).get_all_sequences(256), dtype=torch.int32)
    ra = torch.tensor(SNGBank(pool2, cfg2["sng"]["q"]).get_all_sequences(256), dtype=torch.int32)
    for L, G in ((256, 256), (64, 256), (64, 64), (100, 128), (256, 300), (40, 100)):
        for mode in ("bitrev", "counter", "off"):
            os.environ["SC_OWEN_MODE"] = mode
            out[f"prep_L{L}_G{G}_{mode}"] = K._prepare_rng_prefix(rb, 8, L, G).numpy()
        os.environ.pop("SC_OWEN_MODE", None)
        cum, kt = K.build_enable_tables(ra, rb, 8, L, rng_levels=G)
        out[f"ktab_L{L}_G{G}"] = kt.numpy()
        out[f"cum_L{L}_G{G}"] = cum.numpy()
    np.savez_compressed(os.path.join(HERE, "rng_golden.npz"), **out)
    print("[rng_golden] written", flush=True)


ALL = {
    "rng": case_rng, "edges": case_edges,
    "cfg1": case_cfg1, "cfg3": case_cfg3, "cfg4": case_cfg4, "cfg5": case_cfg5, "cfg2": case_cfg2,
    "configs": case_configs,
}
CASE_NAMES = {
    "rng": ["rng_golden"],
    "cfg1": ["cfg1_lfsr", "cfg1_sobol", "cfg1_unipolar"],
    "cfg2": ["cfg2_slice"], "cfg3": ["cfg3_qk", "cfg3_av"],
    "cfg4": ["cfg4_L256", "cfg4_L128", "cfg4_L64", "cfg4_L128_grid256"],
    "cfg5": ["cfg5_slice"],
    "configs": ["e_cfg_antithetic", "e_cfg_altseed8", "e_cfg_altseed6_prefix", "e_cfg_custom_seed", "e_cfg_dse"],
    "edges": ["e_rowgroup_bip", "e_rowgroup_uni", "e_row_uni_pertensor", "e_row3d_bip", "e_row3d_bip_gt",
              "e_row3d_uni", "e_tensor_uni_small", "e_halve", "e_prefix64", "e_rescale64", "e_rescale_long",
              "e_p4", "e_p6_uni_prefix", "e_chunk_rem", "e_chunk_ge_d", "e_chunk_short", "e_zeros",
              "e_zeros_uni", "e_tiny", "e_head_small", "e_head_prefix", "e_lfsr_indep", "e_lfsr_perelem",
              "e_lfsr_perelem_prefix", "e_truerandom", "e_tensor_lfsr6", "e_owen_counter", "e_owen_off",
              "e_owen_disable", "e_rescale_noscramble", "e_smooth_row", "e_smooth_head"],
}


def main():
    global _POOL
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the reference checkout")
    ap.add_argument("--skip-existing", action="store_true")
    ap.add_argument("cases", nargs="*")
    args = ap.parse_args()
    sys.path.insert(0, REPO)
    _install_reference(args.reference)
    _POOL = mp.get_context("fork").Pool(8)
    wanted = args.cases or [n for v in CASE_NAMES.values() for n in v]
    for grp, fn in ALL.items():
        names = [n for n in CASE_NAMES[grp] if n in wanted]
        if args.skip_existing:
            names = [n for n in names if not os.path.exists(os.path.join(HERE, n + ".npz"))]
        if names:
            fn(set(names))
    _POOL.close()
    _POOL.join()


if __name__ == "__main__":
    main()
