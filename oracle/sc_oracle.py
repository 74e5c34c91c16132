"""CPU oracle for the stochastic-computing matmul -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference ``scmp_kernels`` algorithm for
``sc_matmul`` (swalther06/scmp_kernels). It is the checker the GPU path is
compared with: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg may import it, and never as the thing measured or shipped.

Parity is pinned: ``tests/test_oracle_golden.py`` checks this restatement
against golden vectors produced by running the reference's own ``sc_matmul``
under ``TRITON_INTERPRET=1`` (``tests/golden/gen_golden.py``).

Arithmetic conventions (they decide bit-exactness):
* every float op is IEEE float32 with round-to-nearest-even, one rounding per
  op (no fused multiply-add), which is what the Triton interpreter and torch's
  CPU kernels compute;
* ``rint`` is round-half-to-even (``libdevice.nearbyint`` and ``torch.round``);
* the in-kernel accumulator of the reference holds exact integers
  (``|S| <= D*L < 2**24``), so it is computed here as an int64 sum ``S``.

File:line citations below are relative to the reference repository root.
"""
from __future__ import annotations

import json
import math
import os
import random
from typing import Optional

import numpy as np

f32 = np.float32


# ---------------------------------------------------------------------------
# RNG sequences  (scmp_kernels/sc/rng.py, scmp_kernels/sc/sng.py)
# ---------------------------------------------------------------------------

def lfsr_sequence(seed: int, length: int, taps, n: Optional[int] = None) -> np.ndarray:
    """Fibonacci LFSR: output = register, then shift right and feed the XOR of
    the tapped bits into bit ``length-1`` (rng.py:55-77)."""
    if seed == 0:
        raise ValueError("LFSR seed must be non-zero")
    n = 2 ** length if n is None else n
    reg, out = seed, []
    for _ in range(n):
        out.append(reg)
        fb = 0
        for t in taps:
            fb ^= (reg >> t) & 1
        reg = (reg >> 1) | (fb << (length - 1))
    return np.array(out, dtype=np.int32)


def true_random_sequence(seed: int, length: int, n: Optional[int] = None) -> np.ndarray:
    """Python ``random`` draws in [0, 2**length - 1] after seeding (rng.py:95-113)."""
    n = 2 ** length if n is None else n
    r = random.Random(seed)
    return np.array([r.randint(0, 2 ** length - 1) for _ in range(n)], dtype=np.int32)


def sobol_default_seed(length: int, seed_type: str) -> list:
    """Direction-number seeds of the Q and K Sobol generators (rng.py:156-171)."""
    if seed_type == "k":
        if length == 8:
            return [1, 1, 1, 1, 9, 1, 41, 255]
        s = [1] * length
        if length >= 5:
            s[4] = 9
        if length >= 7:
            s[6] = 41
        return s
    return [1] * length


def sobol_sequence(length: int, seed=None, seed_type: str = "q",
                   n: Optional[int] = None) -> np.ndarray:
    """Gray-code Sobol: emit the value, then XOR direction vector ``V[lsz(i)]``
    where ``V[i] = int(seed[i] / 2**(i+1) * 2**length)`` (rng.py:173-225)."""
    n = 2 ** length if n is None else n
    seed = list(seed) if seed is not None else sobol_default_seed(length, seed_type)
    V = [int(seed[i] / (1 << (i + 1)) * (1 << length)) for i in range(length)]
    val, out = 0, []
    for idx in range(n):
        out.append(val)
        k = 0
        while (idx >> k) & 1:
            k += 1
        if k < length:
            val ^= V[k]
    return np.array(out, dtype=np.int32)


def apply_scramble(seq: np.ndarray, perm) -> np.ndarray:
    """Output bit ``i`` = source bit ``perm[i]`` (sng.py:15-29)."""
    res = np.zeros_like(seq)
    for i, src in enumerate(perm):
        res |= ((seq >> src) & 1) << i
    return res


def _pool_sequence(cfg: dict, sc_prec: int) -> np.ndarray:
    """One RNG of the pool (sng.py:92-98 -> rng.py:242-268)."""
    typ = cfg.get("type", "lfsr")
    if typ == "lfsr":
        return lfsr_sequence(cfg["seed"], sc_prec, cfg["taps"])
    if typ == "true_random":
        return true_random_sequence(cfg["seed"], sc_prec)
    if typ == "sobol":
        return sobol_sequence(sc_prec, cfg.get("seed"), cfg.get("seed_type", "q"))
    raise ValueError(f"Unknown RNG type: {typ}")


def bank_sequences(config: dict, sc_prec: int, which: str) -> np.ndarray:
    """``SNGBank(...).get_all_sequences(2**sc_prec)`` for side ``which`` in
    {"q", "k"} (sng.py:187-230, called from kernels.py:76-85)."""
    n = 2 ** sc_prec
    sngs = config["sng"][which]
    pool = {}
    for s in sngs:
        rid = s["rng_id"]
        if rid not in pool:
            pool[rid] = _pool_sequence(config["rng_pool"][rid], sc_prec)
    out = np.zeros((len(sngs), n), dtype=np.int32)
    for i, s in enumerate(sngs):
        seq = pool[s["rng_id"]]
        sc = s.get("scramble")
        out[i] = apply_scramble(seq, sc) if sc is not None else seq
    return out


def make_sobol_simple_config(q_e: int, k_e: int, sc_prec: int = 8) -> dict:
    """Default config when ``config=None`` (config_helpers.py:583-607)."""
    return {
        "rng_pool": [{"type": "sobol", "seed_type": "q"}, {"type": "sobol", "seed_type": "k"}],
        "sng": {"q": [{"rng_id": 0, "scramble": None} for _ in range(q_e)],
                "k": [{"rng_id": 1, "scramble": None} for _ in range(k_e)]},
    }


# ---------------------------------------------------------------------------
# prefix / Owen scramble / rescale  (scmp_kernels/sc/kernels.py:596-704)
# ---------------------------------------------------------------------------

OWEN_SEED = 0x5A5A5A5A


def resolve_rng_levels(sc_prec: int, rng_levels) -> int:
    """kernels.py:596-606."""
    return 2 ** sc_prec if rng_levels is None else int(rng_levels)


def bit_reverse(x: np.ndarray, n_bits: int) -> np.ndarray:
    """kernels.py:638-643."""
    y = np.zeros_like(x)
    for i in range(n_bits):
        y |= ((x >> i) & 1) << (n_bits - 1 - i)
    return y


def owen_masks(D: int, base_levels: int, env=None) -> Optional[np.ndarray]:
    """Per-dimension XOR masks of ``_owen_scramble`` (kernels.py:646-670), or
    None when scrambling is off. ``env`` defaults to ``os.environ``."""
    env = os.environ if env is None else env
    if env.get("SC_DISABLE_OWEN", "0") == "1":
        return None
    mode = env.get("SC_OWEN_MODE", "bitrev").lower()
    if mode == "off":
        return None
    idx = np.arange(D, dtype=np.int64) % base_levels
    if mode == "counter":
        return idx.astype(np.int32)
    if mode == "bitrev":
        return bit_reverse(idx, int(round(math.log2(base_levels)))).astype(np.int32)
    import torch  # "random": the reference draws the masks with a seeded torch generator
    g = torch.Generator().manual_seed(OWEN_SEED)
    return torch.randint(0, base_levels, (D, 1), generator=g).numpy()[:, 0].astype(np.int32)


def prepare_rng_prefix(rng: np.ndarray, sc_prec: int, stoc_len: int, rng_levels,
                       env=None) -> np.ndarray:
    """kernels.py:673-704: take the first ``stoc_len`` values; on the full grid
    XOR the Owen mask only when truncating; on a resized grid XOR the mask
    (unless SC_SCRAMBLE_RESCALE=0) and rescale with floor(x*G/2**p)."""
    env = os.environ if env is None else env
    G = resolve_rng_levels(sc_prec, rng_levels)
    base = 2 ** sc_prec
    is_prefix = stoc_len < rng.shape[1]
    prefix = rng[:, :stoc_len].copy() if is_prefix else rng.copy()
    if G == base:
        if is_prefix:
            m = owen_masks(prefix.shape[0], base, env)
            if m is not None:
                prefix ^= m[:, None]
        return prefix.astype(np.int32)
    if env.get("SC_SCRAMBLE_RESCALE", "1") == "1":
        m = owen_masks(prefix.shape[0], base, env)
        if m is not None:
            prefix ^= m[:, None]
    return ((prefix.astype(np.int64) * G) // base).astype(np.int32)


# ---------------------------------------------------------------------------
# enable-signal tables  (kernels.py:102-169, 712-759)
# ---------------------------------------------------------------------------

def next_pow2(x: int) -> int:
    return 1 << (int(x) - 1).bit_length()


def k_table(ra: np.ndarray, L: int, V: int) -> np.ndarray:
    """``k_table[d, v] = #{t < L : ra[d, t] < v}`` (kernels.py:140-169)."""
    v = np.arange(V)
    # computed once per distinct sequence row (large D repeats few rows)
    rows, inv = np.unique(np.asarray(ra)[:, :L], axis=0, return_inverse=True)
    kt = (rows[:, :, None] < v[None, None, :]).sum(axis=1).astype(np.int32)
    return kt[np.asarray(inv).reshape(-1)]


def count_table(rb_row: np.ndarray, L: int, V: int) -> np.ndarray:
    """``cum[k, v] = #{i < k : rb[i] < v}`` for one dimension (kernels.py:102-137)."""
    ind = (rb_row[:L, None] < np.arange(V)[None, :]).astype(np.int32)
    cum = np.zeros((L + 1, V), dtype=np.int32)
    np.cumsum(ind, axis=0, out=cum[1:])
    return cum


def enable_sum(kt: np.ndarray, rb: np.ndarray, L: int, ba, bb, sa=None, sb=None) -> np.ndarray:
    """Integer accumulator of ``enable_matmul_tiled_kernel`` (kernels.py:216-245):
    ``S[m,n] = sum_d sa[m,d] sb[n,d] cum_d[k_table[d, ba[m,d]], bb[n,d]]``.
    ``ba`` is (N, D), ``bb`` is (M, D); signs are None for unipolar."""
    N, D = ba.shape
    M = bb.shape[0]
    V = kt.shape[1]
    S = np.zeros((N, M), dtype=np.int64)
    cache = {}
    for d in range(D):
        key = rb[d, :L].tobytes()
        cum = cache.get(key)
        if cum is None:
            cum = count_table(rb[d], L, V)
            cache[key] = cum
        k = kt[d, ba[:, d]]
        c = cum[k[:, None], bb[None, :, d]].astype(np.int64)
        if sa is not None:
            c *= sa[:, d].astype(np.int64)[:, None] * sb[:, d].astype(np.int64)[None, :]
        S += c
    return S


class Tables:
    """RNG sequences plus prepared tables for one (config, sc_prec, stoc_len, G)
    (kernels.py:67-87 and 762-777)."""

    def __init__(self, config: dict, sc_prec: int, stoc_len: int, rng_levels, env=None):
        G = resolve_rng_levels(sc_prec, rng_levels)
        self.G, self.L = G, stoc_len
        self.V = next_pow2(G + 1)
        qa = bank_sequences(config, sc_prec, "q")
        kb = bank_sequences(config, sc_prec, "k")
        self.ra = prepare_rng_prefix(qa, sc_prec, stoc_len, G, env)
        self.rb = prepare_rng_prefix(kb, sc_prec, stoc_len, G, env)
        self.kt = k_table(self.ra, stoc_len, self.V)

    def S(self, ba, bb, sa=None, sb=None, d_off: int = 0):
        D = ba.shape[1]
        return enable_sum(self.kt[d_off:d_off + D], self.rb[d_off:d_off + D], self.L, ba, bb, sa, sb)


def scaled(S: np.ndarray, q_max: int, L: int) -> np.ndarray:
    """``acc *= q_max_sq / stoc_len`` (kernels.py:212, 248)."""
    inner = f32(q_max * q_max) / f32(L)
    return S.astype(f32) * inner


# ---------------------------------------------------------------------------
# quantisation recipes  (scmp_kernels/quant/fused.py, quant/grouped.py)
# ---------------------------------------------------------------------------

def _sign_i8(xc: np.ndarray) -> np.ndarray:
    return np.where(xc > 0, 1, np.where(xc < 0, -1, 0)).astype(np.int8)


def fused_quantize_bipolar(x: np.ndarray, abs_max: float, sc_prec: int, G: int):
    """fused.py:162-189 with the flat kernel variant (fused.py:86-112)."""
    q = 2 ** (sc_prec - 1) - 1
    abs_max = max(abs_max, 1e-5)
    scale = abs_max / q
    inv = f32(1.0 / scale)
    xc = np.clip(np.rint(x * inv), f32(-q), f32(q))
    ratio = f32(G) / f32(q)
    boundary = np.rint(np.abs(xc) * ratio).astype(np.int16)
    return boundary, _sign_i8(xc), scale


def fused_quantize_bipolar_perrow(x: np.ndarray, sc_prec: int, G: int):
    """fused.py:134-159 with the per-row kernel variant (fused.py:65-81)."""
    q = 2 ** (sc_prec - 1) - 1
    am = np.maximum(np.abs(x).max(axis=1), f32(1e-5)) if x.shape[1] else np.full(x.shape[0], f32(1e-5))
    scale = (am / f32(q)).astype(f32)
    inv = (f32(1.0) / scale).astype(f32)
    xc = np.clip(np.rint(x * inv[:, None]), f32(-q), f32(q))
    ratio = f32(G) / f32(q)
    boundary = np.rint(np.abs(xc) * ratio).astype(np.int16)
    return boundary, _sign_i8(xc), scale


def fused_quantize_unipolar(x: np.ndarray, fp_max: float, fp_min: float, sc_prec: int, G: int):
    """fused.py:192-223 (compute_sum=True, the per-row kernel variant with the
    host scale and zero point, fused.py:82-84 and 113-121)."""
    q = 2 ** sc_prec - 1
    rng_fp = max(fp_max - fp_min, 1e-5)
    scale = rng_fp / q
    inv = f32(1.0 / scale)
    zp = round(-fp_min / scale)
    zp = max(0, min(q, zp))
    zpf = f32(float(zp))
    xc = np.clip(np.rint((x * inv) + zpf), f32(0), f32(q))
    ratio = f32(G) / f32(q)
    boundary = np.rint(xc * ratio).astype(np.int32)
    row_sum = xc.sum(axis=1, dtype=np.float64).astype(f32)  # exact: integers < 2**24
    return boundary, scale, float(zp), row_sum


def fused_quant_bipolar_batched(x: np.ndarray, inv_scale: np.ndarray, sc_prec: int, G: int):
    """fused.py:237-283 (x is (BH, rows, cols); output kept in (BH, rows, cols)
    order here -- the reference's transposed store is only a layout)."""
    q = 2 ** (sc_prec - 1) - 1
    qmin = -(2 ** (sc_prec - 1))
    xc = np.clip(np.rint(x * inv_scale[:, None, None]), f32(qmin), f32(q))
    ratio = f32(G) / f32(q)
    boundary = np.rint(np.abs(xc) * ratio).astype(np.int16)
    return boundary, _sign_i8(xc)


def _groups(rows: int, G: int):
    """Row groups of ``_grouped_*_quant``: full groups of G then one remainder
    group; G >= rows is a single group (grouped.py:28-75)."""
    if G >= rows:
        return [(0, rows)]
    out = [(i * G, (i + 1) * G) for i in range(rows // G)]
    if rows % G:
        out.append(((rows // G) * G, rows))
    return out


def grouped_symmetric_quant(x: np.ndarray, G: int, q: int):
    """grouped.py:13-75: scale = clamp(absmax_g, 1e-5)/q, x_int =
    clamp(round(x/scale), +-q), sign with 0 -> +1."""
    rows = x.shape[0]
    scale_row = np.zeros(rows, dtype=f32)
    for r0, r1 in _groups(rows, G):
        am = np.maximum(np.abs(x[r0:r1]).max() if x[r0:r1].size else f32(0), f32(1e-5))
        scale_row[r0:r1] = f32(am) / f32(q)
    xi = np.clip(np.rint(x / scale_row[:, None]), f32(-q), f32(q)).astype(f32)
    sign = np.sign(xi).astype(np.int8)
    sign[sign == 0] = 1
    return scale_row, xi, sign


def grouped_asymmetric_quant(x: np.ndarray, G: int, q: int):
    """grouped.py:78-133: scale = clamp(max-min, 1e-5)/q, zp =
    clamp(round(-min/scale), 0, q), x_int = clamp(round(x/scale + zp), 0, q)."""
    rows = x.shape[0]
    scale_row = np.zeros(rows, dtype=f32)
    zp_row = np.zeros(rows, dtype=f32)
    for r0, r1 in _groups(rows, G):
        mx, mn = x[r0:r1].max(), x[r0:r1].min()
        rg = np.maximum(f32(mx - mn), f32(1e-5))
        sc = f32(rg) / f32(q)
        scale_row[r0:r1] = sc
        zp_row[r0:r1] = np.clip(np.rint(f32(-mn) / sc), f32(0), f32(q))
    xi = np.clip(np.rint((x / scale_row[:, None]) + zp_row[:, None]), f32(0), f32(q)).astype(f32)
    return scale_row, zp_row, xi


def grouped_symmetric_quant_batched(x: np.ndarray, G: int, q: int):
    """grouped.py:136-163 (G == 1 or G >= rows)."""
    BH, rows, cols = x.shape
    if G >= rows:
        am = np.maximum(np.abs(x).reshape(BH, -1).max(axis=1), f32(1e-5))
        scale = (am / f32(q)).astype(f32)
        xi = np.clip(np.rint(x / scale[:, None, None]), f32(-q), f32(q)).astype(f32)
        scale_r = np.repeat(scale[:, None], rows, axis=1)
    elif G == 1:
        am = np.maximum(np.abs(x).max(axis=2), f32(1e-5))
        scale_r = (am / f32(q)).astype(f32)
        xi = np.clip(np.rint(x / scale_r[:, :, None]), f32(-q), f32(q)).astype(f32)
    else:
        raise NotImplementedError(f"_grouped_symmetric_quant_batched: G={G} not supported (use G=1 or G>=rows)")
    sign = np.sign(xi).astype(np.int8)
    sign[sign == 0] = 1
    return scale_r, xi, sign


def _bound_div(xi_abs: np.ndarray, G: int, q: int) -> np.ndarray:
    """``(x_int.abs() * max_rng_val / q_max).round().short()`` (kernels.py:1679-1680)."""
    return np.rint((xi_abs * f32(G)) / f32(q)).astype(np.int16)


def smooth(a: np.ndarray, b: np.ndarray, s: np.ndarray):
    """``apply_smoothing``: (a / s, b * s) along D (smoothquant.py:96-126)."""
    s = s.astype(f32)
    return (a / s).astype(f32), (b * s).astype(f32)


# ---------------------------------------------------------------------------
# path orchestrators  (scmp_kernels/sc/kernels.py, scmp_kernels/sc/matmul.py)
# ---------------------------------------------------------------------------

_TABLES_CACHE: dict = {}


def _tables(config, D, sc_prec, stoc_len, G, env):
    """Tables of one key, kept like the reference's RNG and table caches
    (kernels.py:59-87, 762-777), with the environment in the key."""
    if config is None:
        config = make_sobol_simple_config(D, D, sc_prec)
    key = (json.dumps(config, sort_keys=True), sc_prec, stoc_len, G,
           json.dumps(env if env is not None else dict(os.environ), sort_keys=True))
    t = _TABLES_CACHE.get(key)
    if t is None:
        t = _TABLES_CACHE[key] = Tables(config, sc_prec, stoc_len, G, env)
    return t


def per_tensor(a, b, mode, sc_prec, config, stoc_len, rng_levels, env=None):
    """``_sc_matmul_per_tensor`` + ``_sc_matmul_enable_triton`` (kernels.py:1053-1204)
    with the host-side ranges of matmul.py:227-230."""
    if a.ndim == 3:
        return np.stack([per_tensor_2d(a[i], b[i], float(a.max()), float(a.min()), float(b.max()),
                                       float(b.min()), mode, sc_prec, config, stoc_len, rng_levels, env)
                         for i in range(a.shape[0])])
    return per_tensor_2d(a, b, float(a.max()), float(a.min()), float(b.max()), float(b.min()),
                         mode, sc_prec, config, stoc_len, rng_levels, env)


def per_tensor_2d(a, b, amax, amin, bmax, bmin, mode, sc_prec, config, stoc_len, rng_levels, env=None):
    N, D = a.shape
    G = resolve_rng_levels(sc_prec, rng_levels)
    T = _tables(config, D, sc_prec, stoc_len, G, env)
    if mode == "bipolar":
        q = 2 ** (sc_prec - 1) - 1
        ba, sa, sca = fused_quantize_bipolar(a, max(abs(amax), abs(amin), 1e-5), sc_prec, G)
        bb, sb, scb = fused_quantize_bipolar(b, max(abs(bmax), abs(bmin), 1e-5), sc_prec, G)
        raw = scaled(T.S(ba, bb, sa, sb), q, stoc_len)
        return raw * f32(sca * scb)
    q = 2 ** sc_prec - 1
    ba, sca, zpa, asum = fused_quantize_unipolar(a, amax, amin, sc_prec, G)
    bb, scb, zpb, bsum = fused_quantize_unipolar(b, bmax, bmin, sc_prec, G)
    raw = scaled(T.S(ba, bb), q, stoc_len)
    t1 = f32(-zpb) * asum[:, None]
    t2 = f32(zpa) * bsum[None, :]
    corr = (t1 - t2) + f32(D * zpa * zpb)
    return (raw + corr) * f32(sca * scb)


def per_row_2d(a, b, group_a, group_b, mode, sc_prec, config, stoc_len, rng_levels, env=None):
    """``_sc_matmul_per_row`` + ``_sc_matmul_grouped_enable`` (kernels.py:1573-1707)."""
    N, D = a.shape
    G = resolve_rng_levels(sc_prec, rng_levels)
    T = _tables(config, D, sc_prec, stoc_len, G, env)
    if mode == "bipolar":
        q = 2 ** (sc_prec - 1) - 1
        sca, ai, sa = grouped_symmetric_quant(a, group_a, q)
        scb, bi, sb = grouped_symmetric_quant(b, group_b, q)
        raw = scaled(T.S(_bound_div(np.abs(ai), G, q), _bound_div(np.abs(bi), G, q), sa, sb), q, stoc_len)
        return raw * (sca[:, None] * scb[None, :])
    q = 2 ** sc_prec - 1
    sca, zpa, ai = grouped_asymmetric_quant(a, group_a, q)
    scb, zpb, bi = grouped_asymmetric_quant(b, group_b, q)
    raw = scaled(T.S(_bound_div(ai, G, q), _bound_div(bi, G, q)), q, stoc_len)
    asum = ai.sum(axis=1, dtype=np.float64).astype(f32)
    bsum = bi.sum(axis=1, dtype=np.float64).astype(f32)
    t1 = (-zpb[None, :]) * asum[:, None]
    t2 = zpa[:, None] * bsum[None, :]
    t4 = (f32(D) * zpa[:, None]) * zpb[None, :]
    raw = raw + ((t1 - t2) + t4)
    return raw * (sca[:, None] * scb[None, :])


def per_row_batched(a, b, group_a, group_b, mode, sc_prec, config, stoc_len, rng_levels, env=None):
    """``_sc_matmul_per_row_batched`` (kernels.py:1778-1895)."""
    BH, M, D = a.shape
    if config is None:
        config = make_sobol_simple_config(D, D, sc_prec)
    if mode == "unipolar":
        return np.stack([per_row_2d(a[i], b[i], group_a, group_b, mode, sc_prec, config, stoc_len,
                                    rng_levels, env) for i in range(BH)])
    G = resolve_rng_levels(sc_prec, rng_levels)
    T = Tables(config, sc_prec, stoc_len, G, env)
    q = 2 ** (sc_prec - 1) - 1
    sca, ai, sa = grouped_symmetric_quant_batched(a, group_a, q)
    scb, bi, sb = grouped_symmetric_quant_batched(b, group_b, q)
    ratio = f32(G / q)
    ba = np.rint(np.abs(ai) * ratio).astype(np.int16)
    bb = np.rint(np.abs(bi) * ratio).astype(np.int16)
    out = []
    inner = (f32(q * q) / f32(stoc_len)) * f32(1.0)
    for i in range(BH):
        raw = T.S(ba[i], bb[i], sa[i], sb[i]).astype(f32) * inner
        out.append(raw * (sca[i][:, None] * scb[i][None, :]))
    return np.stack(out)


def per_row_chunked(a, b, sc_prec, config, chunk_d, stoc_len, rng_levels, env=None):
    """``_sc_matmul_per_row_mlp`` fast path + ``_sc_matmul_bipolar_mlp_chunked``
    (kernels.py:1500-1520, 1274-1383): per chunk of ``chunk_d`` columns a
    per-row quant, then ``out += fl32(S_c * inner) * (sa_c x sb_c)``; every
    chunk reuses table rows 0..chunk_d-1."""
    N, D = a.shape
    M = b.shape[0]
    G = resolve_rng_levels(sc_prec, rng_levels)
    if config is None:
        config = make_sobol_simple_config(chunk_d, chunk_d, sc_prec)
    T = Tables(config, sc_prec, stoc_len, G, env)
    q = 2 ** (sc_prec - 1) - 1
    out = np.zeros((N, M), dtype=f32)
    for d0 in range(0, D, chunk_d):
        d1 = min(d0 + chunk_d, D)
        ba, sa, sca = fused_quantize_bipolar_perrow(np.ascontiguousarray(a[:, d0:d1]), sc_prec, G)
        bb, sb, scb = fused_quantize_bipolar_perrow(np.ascontiguousarray(b[:, d0:d1]), sc_prec, G)
        part = scaled(T.S(ba, bb, sa, sb, d_off=0), q, stoc_len)
        out = out + part * (sca[:, None] * scb[None, :])
    return out


def per_head(a, b, sc_prec, config, stoc_len, rng_levels, env=None):
    """matmul.py:264-279 + ``_sc_matmul_per_head_bipolar`` (kernels.py:440-585)."""
    BH, N, D = a.shape
    BHk, M, Dk = b.shape
    if BHk != BH or Dk != D:
        raise ValueError(
            f"_sc_matmul_per_head_bipolar: shape mismatch — q is (BH={BH}, N={N}, D={D}), "
            f"k is (BH={BHk}, M={M}, D={Dk}); require equal BH and D.")
    if config is None:
        config = make_sobol_simple_config(D, D, sc_prec)
    G = resolve_rng_levels(sc_prec, rng_levels)
    T = Tables(config, sc_prec, stoc_len, G, env)
    q = 2 ** (sc_prec - 1) - 1

    def head_scale(x):
        mx = x.reshape(BH, -1).max(axis=1)
        mn = x.reshape(BH, -1).min(axis=1)
        am = np.maximum(np.maximum(np.abs(mx), np.abs(mn)), f32(1e-5)).astype(f32)
        sc = (am / f32(q)).astype(f32)
        return sc, (f32(1.0) / sc).astype(f32)

    sq, iq = head_scale(a)
    sk, ik = head_scale(b)
    ba, sa = fused_quant_bipolar_batched(a, iq, sc_prec, G)
    bb, sb = fused_quant_bipolar_batched(b, ik, sc_prec, G)
    inner = f32(q * q) / f32(stoc_len)
    hs = (sq * sk).astype(f32)
    return np.stack([T.S(ba[i], bb[i], sa[i], sb[i]).astype(f32) * (inner * hs[i]) for i in range(BH)])


_GRAN = ("per_tensor", "per_row", "per_head")
_MODES = ("bipolar", "unipolar")


def sc_matmul(a, b, granularity="per_row", *, mode="bipolar", sc_prec=8, stoc_len=None, chunk_d=0,
              group_a=1, group_b=1, rng_levels=None, config=None, halve_bipolar_stoc_len=False,
              smooth_scales=None, env=None):
    """``_sc_matmul_impl`` dispatch (matmul.py:81-279) on float32 numpy arrays."""
    a = np.asarray(a, dtype=f32)
    b = np.asarray(b, dtype=f32)
    if granularity not in _GRAN:
        raise ValueError(f"sc_matmul: unknown granularity '{granularity}'. Expected one of {_GRAN}.")
    if mode not in _MODES:
        raise ValueError(f"sc_matmul: unknown mode '{mode}'. Expected one of {_MODES}.")
    if halve_bipolar_stoc_len and mode == "bipolar":
        h = 2 ** (sc_prec - 1)
        stoc_len = h if stoc_len is None else stoc_len
        rng_levels = h if rng_levels is None else rng_levels
    if smooth_scales is not None:
        a, b = smooth(a, b, np.asarray(smooth_scales, dtype=f32))
    if stoc_len is None:
        stoc_len = 2 ** sc_prec
    if isinstance(config, str):
        config = json.loads(config)
    if granularity == "per_tensor":
        return per_tensor(a, b, mode, sc_prec, config, stoc_len, rng_levels, env)
    if granularity == "per_row":
        if chunk_d > 0 and mode == "bipolar" and a.ndim == 2 and a.shape[1] > chunk_d:
            return per_row_chunked(a, b, sc_prec, config, chunk_d, stoc_len, rng_levels, env)
        if a.ndim == 3:
            return per_row_batched(a, b, group_a, group_b, mode, sc_prec, config, stoc_len, rng_levels, env)
        return per_row_2d(a, b, group_a, group_b, mode, sc_prec, config, stoc_len, rng_levels, env)
    return per_head(a, b, sc_prec, config, stoc_len, rng_levels, env)
