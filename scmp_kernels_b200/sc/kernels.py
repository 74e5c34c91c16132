"""Host orchestration of the B200 SC-GEMM: RNG/table cache and path entry points.

Mirrors the module ``scmp_kernels.sc.kernels`` (scmp_kernels/sc/kernels.py):
the same private path functions (``_sc_matmul_per_tensor``,
``_sc_matmul_per_row``, ``_sc_matmul_per_row_mlp``,
``_sc_matmul_per_row_batched``, ``_sc_matmul_per_head_bipolar``), the same
cache semantics and ``clear_rng_cache`` / ``det_kernel_tuning``. Every path
ends in one call of the native ``scmp_sc_matmul`` (quantisation, SC-GEMM and
float epilogue on the device, no host synchronisation).

Enable tables. The reference builds, per RNG config, ``k_table[d][v]`` and the
int16 ``cum_indicator[d][k][v]`` (1.08 GB at D=4096, L=256). Here the prepared
sequences (prefix / Owen scramble / rescale, restated from kernels.py:596-704)
are deduplicated to their distinct rows and the device keeps, per distinct
row, ``ktab[v]`` and the bit-packed comparator stream ``[rb[t] < v]`` for every
boundary ``v``; ``cum_indicator[k][v]`` is the popcount of its first ``k``
bits. Under the default Sobol config every dimension shares one row, so the
tables are a few KB.
"""
from __future__ import annotations

import contextlib
import ctypes
import json
import math
import os
import threading
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from .. import _lib
from ..quant.smoothquant import apply_smoothing, _check_smoothing
from .sng import RNGPool, SNGBank

# ---------------------------------------------------------------------------
# RNG sequences and prepared tables
# ---------------------------------------------------------------------------

_rng_seq_cache: dict[str, tuple[np.ndarray, np.ndarray]] = {}
_enable_table_cache: dict[str, "EnableTables"] = {}
_k_table_cache: dict = {}  # kept for API parity; tables live in _enable_table_cache

_OWEN_SCRAMBLE_SEED = 0x5A5A5A5A


def _config_cache_key(config: dict, sc_prec: int, device) -> str:
    """kernels.py:62-64."""
    return json.dumps(config, sort_keys=True) + f"|{sc_prec}|{device}"


def _get_cached_sequences(config: dict, sc_prec: int, device) -> tuple[np.ndarray, np.ndarray]:
    """Host int32 sequences ``(q_e, 2**p)`` and ``(k_e, 2**p)`` (kernels.py:67-87)."""
    key = _config_cache_key(config, sc_prec, device)
    if key not in _rng_seq_cache:
        n = 2 ** sc_prec
        pool = RNGPool(config["rng_pool"], sc_prec)
        qa = np.ascontiguousarray(SNGBank(pool, config["sng"]["q"]).get_all_sequences(n), dtype=np.int32)
        kb = np.ascontiguousarray(SNGBank(pool, config["sng"]["k"]).get_all_sequences(n), dtype=np.int32)
        _rng_seq_cache[key] = (qa, kb)
    return _rng_seq_cache[key]


def clear_rng_cache():
    """Drop cached RNG sequences and enable tables (kernels.py:90-95)."""
    _rng_seq_cache.clear()
    _enable_table_cache.clear()
    _k_table_cache.clear()


def _resolve_rng_levels(sc_prec: int, rng_levels: Optional[int]) -> int:
    """kernels.py:596-606."""
    return 2 ** sc_prec if rng_levels is None else int(rng_levels)


def _bit_reverse(x: np.ndarray, n_bits: int) -> np.ndarray:
    y = np.zeros_like(x)
    for i in range(n_bits):
        y |= ((x >> i) & 1) << (n_bits - 1 - i)
    return y


def _owen_masks(D: int, base_levels: int, device) -> Optional[np.ndarray]:
    """Per-dimension XOR masks (kernels.py:646-670); None when scrambling is off.
    The "random" family draws from a seeded torch generator on ``device``,
    exactly as the reference does."""
    if os.environ.get("SC_DISABLE_OWEN", "0") == "1":
        return None
    mode = os.environ.get("SC_OWEN_MODE", "bitrev").lower()
    if mode == "off":
        return None
    idx = np.arange(D, dtype=np.int64) % base_levels
    if mode == "counter":
        return idx.astype(np.int32)
    if mode == "bitrev":
        return _bit_reverse(idx, int(round(math.log2(base_levels)))).astype(np.int32)
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(_OWEN_SCRAMBLE_SEED)
    m = torch.randint(0, base_levels, (D, 1), generator=g, device=dev)
    return m[:, 0].to(torch.int32).cpu().numpy()


def _prepare_rng_prefix(rng: np.ndarray, sc_prec: int, stoc_len: int, rng_levels, device="cpu"):
    """Prefix, Owen scramble and rescale of one operand's sequences (kernels.py:673-704)."""
    G = _resolve_rng_levels(sc_prec, rng_levels)
    base = 2 ** sc_prec
    is_prefix = stoc_len < rng.shape[1]
    prefix = np.array(rng[:, :stoc_len] if is_prefix else rng, dtype=np.int64)
    if G == base:
        if is_prefix:
            m = _owen_masks(prefix.shape[0], base, device)
            if m is not None:
                prefix ^= m[:, None]
        return prefix.astype(np.int32)
    if os.environ.get("SC_SCRAMBLE_RESCALE", "1") == "1":
        m = _owen_masks(prefix.shape[0], base, device)
        if m is not None:
            prefix ^= m[:, None]
    return ((prefix * G) // base).astype(np.int32)


def _next_pow2(x: int) -> int:
    return 1 << (int(x) - 1).bit_length()


@dataclass
class EnableTables:
    """Device-resident enable tables of one (config, sc_prec, stoc_len, grid)."""
    ktab: torch.Tensor      # (rows_a, vcap+1) int16
    pattern: torch.Tensor   # (rows_b, vcap+1, lp/32) int32 (bit-packed streams)
    pattern4: torch.Tensor  # the same streams in the e2m1-sliced bit order
    amap: torch.Tensor      # (config q_e,) int32: dimension -> ktab row
    bmap: torch.Tensor      # (config k_e,) int32: dimension -> pattern row
    L: int
    lp: int
    G: int
    vcap: int
    n_dims: int             # dimensions the config describes (min of q_e, k_e)

    def maps_for(self, D: int, period: Optional[int] = None):
        """Row maps for ``D`` dimensions; with ``period`` dimension ``j`` uses
        config row ``j % period`` (the chunked path reuses rows 0..chunk_d-1)."""
        if period is None:
            if D > self.n_dims:
                raise ValueError(
                    f"sc_matmul: the RNG config describes {self.n_dims} elements per operand but "
                    f"D={D}; the reference would read past its sequence table")
            return self.amap[:D], self.bmap[:D]
        if period > self.n_dims:
            raise ValueError(
                f"sc_matmul: the RNG config describes {self.n_dims} elements but chunk_d={period}")
        idx = torch.arange(D, device=self.amap.device) % period
        return self.amap[idx].contiguous(), self.bmap[idx].contiguous()


def build_enable_tables(config: dict, sc_prec: int, device, stoc_len: Optional[int] = None,
                        rng_levels: Optional[int] = None) -> EnableTables:
    """Build the device tables for one key (replaces kernels.py:712-759)."""
    if stoc_len is None:
        stoc_len = 2 ** sc_prec
    if stoc_len > 2 ** sc_prec:
        raise ValueError(
            f"sc_matmul: stoc_len={stoc_len} exceeds the 2**sc_prec={2 ** sc_prec} values of the "
            "RNG sequences (the reference would index past each sequence row)")
    G = _resolve_rng_levels(sc_prec, rng_levels)
    qa, kb = _get_cached_sequences(config, sc_prec, device)
    ra = _prepare_rng_prefix(qa, sc_prec, stoc_len, G, device)
    rb = _prepare_rng_prefix(kb, sc_prec, stoc_len, G, device)
    ua, ia = np.unique(ra, axis=0, return_inverse=True)
    ub, ib = np.unique(rb, axis=0, return_inverse=True)
    vmax = max(int(ra.max(initial=0)), int(rb.max(initial=0)))
    vcap = max(G, vmax + 1)
    if vcap > 32767:
        raise ValueError(f"sc_matmul: enable grid of {vcap} levels is not supported (max 32767)")
    lp = max(32, _next_pow2(stoc_len))
    dev = torch.device(device)
    ua_t = torch.from_numpy(np.ascontiguousarray(ua, dtype=np.int32)).to(dev)
    ub_t = torch.from_numpy(np.ascontiguousarray(ub, dtype=np.int32)).to(dev)
    ktab = torch.empty((ua.shape[0], vcap + 1), dtype=torch.int16, device=dev)
    pattern = torch.empty((ub.shape[0], vcap + 1, lp // 32), dtype=torch.int32, device=dev)
    pattern4 = torch.empty_like(pattern)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().scmp_build_tables(
            ua_t.data_ptr(), ua.shape[0], ub_t.data_ptr(), ub.shape[0], stoc_len, lp, vcap,
            ktab.data_ptr(), pattern.data_ptr(), pattern4.data_ptr(),
            ctypes.c_void_p(_lib.stream_handle(dev))),
            "build_enable_tables")
    amap = torch.from_numpy(np.asarray(ia, dtype=np.int32).reshape(-1)).to(dev)
    bmap = torch.from_numpy(np.asarray(ib, dtype=np.int32).reshape(-1)).to(dev)
    return EnableTables(ktab, pattern, pattern4, amap, bmap, stoc_len, lp, G, vcap,
                        min(ra.shape[0], rb.shape[0]))


# The default config (config=None) of each (D, sc_prec), built once with its
# JSON key: it is deterministic, private to this module and never mutated,
# so a call with config=None skips serialising a D-element config.
_DEFAULT_CONFIGS: dict = {}   # (D, sc_prec) -> config dict
_DEFAULT_KEYS: dict = {}      # id(config dict) -> json.dumps(config, sort_keys=True)


def _enable_table_cache_key(config: dict, sc_prec: int, device) -> str:
    base = _DEFAULT_KEYS.get(id(config))
    if base is None or _DEFAULT_CONFIGS.get(base[1]) is not config:
        enc = json.dumps(config, sort_keys=True)
    else:
        enc = base[0]
    return enc + f"|{sc_prec}|{device}|enable"


def _get_cached_enable_tables(config: dict, sc_prec: int, device, stoc_len: Optional[int] = None,
                              rng_levels: Optional[int] = None) -> EnableTables:
    """kernels.py:762-777 (keyed by config, precision, device, stream length and
    grid; like the reference, not by the Owen environment variables)."""
    if stoc_len is None:
        stoc_len = 2 ** sc_prec
    G = _resolve_rng_levels(sc_prec, rng_levels)
    key = _enable_table_cache_key(config, sc_prec, device) + f"|sl={stoc_len}|rng={G}"
    t = _enable_table_cache.get(key)
    if t is None:
        t = build_enable_tables(config, sc_prec, device, stoc_len, G)
        _enable_table_cache[key] = t
    return t


# ---------------------------------------------------------------------------
# det_kernel_tuning (kernels.py:1728-1745): a tile-shape switch in the
# reference; the integers and floats it produces are the same either way, so
# here it only counts nesting.
# ---------------------------------------------------------------------------

_DET_KERNEL_TUNING_DEPTH = 0


class det_kernel_tuning:
    """Re-entrant context manager kept for API compatibility."""

    def __enter__(self):
        global _DET_KERNEL_TUNING_DEPTH
        _DET_KERNEL_TUNING_DEPTH += 1
        return self

    def __exit__(self, *_):
        global _DET_KERNEL_TUNING_DEPTH
        _DET_KERNEL_TUNING_DEPTH -= 1


def _det_kernel_tuning_active() -> bool:
    return _DET_KERNEL_TUNING_DEPTH > 0


# ---------------------------------------------------------------------------
# native launch
# ---------------------------------------------------------------------------

_FORCE_SIMT = os.environ.get("SCMP_FORCE_SIMT", "0") == "1"


_REDIRECT = threading.local()


@contextlib.contextmanager
def output_to(peers, offset: int, ld: int, result: torch.Tensor, self_index: int = -1):
    """Within the block, every sc_matmul launch of this thread stores its
    (batch, n, m) result at element ``offset + (h*n + i)*ld + j`` of each device
    pointer in ``peers`` (the multi-GPU all-gather fused into the GEMM's
    epilogue) and returns ``result`` instead of a new tensor. ``self_index``:
    the entry of ``peers`` in this device's memory, if any (the GEMM then
    stores each tile there first and copies it to the others while the next
    tile computes)."""
    if not 1 <= len(peers) <= _lib.MAX_OUT_PEERS:
        raise ValueError(f"output_to: 1..{_lib.MAX_OUT_PEERS} destinations, got {len(peers)}")
    if not -1 <= self_index < len(peers):
        raise ValueError(f"output_to: self_index {self_index} outside the destinations")
    prev = getattr(_REDIRECT, "value", None)
    _REDIRECT.value = ((ctypes.c_void_p * len(peers))(*peers), len(peers), int(offset), int(ld), result,
                       int(self_index))
    try:
        yield
    finally:
        _REDIRECT.value = prev


def _to_host(y: torch.Tensor) -> torch.Tensor:
    """The result for host operands: copied into page-locked host memory (the
    caching host allocator reuses it across calls), which transfers at the
    full link rate, unlike a fresh pageable tensor that is faulted in page by
    page during a synchronous copy."""
    out = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
    out.copy_(y, non_blocking=True)
    torch.cuda.current_stream(y.device).synchronize()
    return out


def _to_device(x: torch.Tensor) -> torch.Tensor:
    if x.device.type != "cuda":
        _lib.require_cuda()
        x = x.cuda()
    return x.float().contiguous()


def _launch(gran: int, mode: str, a: torch.Tensor, b: torch.Tensor, sc_prec: int, tables: EnableTables,
            *, group_a=1, group_b=1, chunk_d=0, smooth: Optional[torch.Tensor] = None,
            period: Optional[int] = None, out: Optional[torch.Tensor] = None,
            workspace: Optional[torch.Tensor] = None, flags: int = 0,
            ranges: Optional[torch.Tensor] = None, b_ready: bool = False,
            workspace_out: Optional[list] = None) -> torch.Tensor:
    """One ``scmp_sc_matmul`` call. a: (batch, n, d) or (n, d); b likewise."""
    three_d = a.dim() == 3
    batch = a.shape[0] if three_d else 1
    n, d = a.shape[-2], a.shape[-1]
    m = b.shape[-2]
    dev = a.device
    redirect = getattr(_REDIRECT, "value", None)
    if redirect is not None:
        peers, n_peers, out_offset, out_ld, out, self_index = redirect
    elif out is None:
        out = torch.empty((batch, n, m) if three_d else (n, m), dtype=torch.float32, device=dev)
    amap, bmap = tables.maps_for(d, period)
    desc = _lib.MatmulDesc(
        granularity=gran, mode=_lib.BIPOLAR if mode == "bipolar" else _lib.UNIPOLAR,
        sc_prec=sc_prec, stoc_len=tables.L, rng_levels=tables.G, chunk_d=chunk_d,
        group_a=group_a, group_b=group_b, batch=batch, n=n, m=m, d=d,
        a=a.data_ptr(), b=b.data_ptr(), smooth_scales=smooth.data_ptr() if smooth is not None else None,
        out=out.data_ptr(), ktab=tables.ktab.data_ptr(), pattern=tables.pattern.data_ptr(),
        pattern4=tables.pattern4.data_ptr(),
        amap=amap.data_ptr(), bmap=bmap.data_ptr(), vcap=tables.vcap, lp=tables.lp,
        flags=flags | (_lib.FLAG_FORCE_SIMT if _FORCE_SIMT else 0),
        tensor_ranges=ranges.data_ptr() if ranges is not None else None)
    if redirect is not None:
        desc.out = None
        desc.out_peers = ctypes.cast(peers, ctypes.c_void_p)
        desc.n_out_peers, desc.out_offset, desc.out_ld = n_peers, out_offset, out_ld
        desc.out_self = self_index + 1
    L = _lib.lib()
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(L.scmp_sc_matmul_workspace_size(ctypes.byref(desc), ctypes.byref(ws_bytes)), "sc_matmul")
    if workspace is None or workspace.numel() < ws_bytes.value:
        workspace = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=dev)
        b_ready = False  # a new workspace holds no quantised b
    if b_ready:  # b's quantised operand is in `workspace` from an earlier call
        desc.flags |= _lib.FLAG_B_READY
    if workspace_out is not None:
        workspace_out.append(workspace)
    _lib.check(L.scmp_sc_matmul(ctypes.byref(desc), ctypes.c_void_p(workspace.data_ptr()),
                                ws_bytes.value, ctypes.c_void_p(_lib.stream_handle(dev))), "sc_matmul")
    return out


def enable_matmul(tables: EnableTables, boundary_a: torch.Tensor, boundary_b: torch.Tensor,
                  sign_a: Optional[torch.Tensor], sign_b: Optional[torch.Tensor], N: int, M: int, D: int,
                  stoc_len: int, q_max_sq: float, is_bipolar: bool, flags: int = 0) -> torch.Tensor:
    """Enable-signal matmul on already-quantised operands (the counterpart of
    enable_matmul_triton, kernels.py:798-868, with this package's tables in
    place of cum_indicator / k_table): boundary (N, D) / (M, D) int16, sign
    int8 (bipolar only); returns (N, M) float32 fl32(S * fl32(q_max_sq / L))."""
    if stoc_len != tables.L:
        raise ValueError(f"enable_matmul: tables are for stoc_len={tables.L}, got {stoc_len}")
    dev = boundary_a.device
    ba = boundary_a.to(torch.int16).contiguous()
    bb = boundary_b.to(torch.int16).contiguous()
    sa = sign_a.to(torch.int8).contiguous() if is_bipolar else None
    sb = sign_b.to(torch.int8).contiguous() if is_bipolar else None
    amap, bmap = tables.maps_for(D)
    out = torch.empty((N, M), dtype=torch.float32, device=dev)
    L = _lib.lib()
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(L.scmp_enable_matmul_workspace_size(N, M, D, ctypes.byref(ws_bytes)), "enable_matmul")
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=dev)
    _lib.check(L.scmp_enable_matmul(
        tables.ktab.data_ptr(), tables.pattern.data_ptr(), amap.data_ptr(), bmap.data_ptr(), tables.vcap,
        tables.L, tables.lp, ba.data_ptr(), bb.data_ptr(), sa.data_ptr() if sa is not None else None,
        sb.data_ptr() if sb is not None else None, N, M, D, float(q_max_sq), 1 if is_bipolar else 0,
        out.data_ptr(), ws.data_ptr(), ws_bytes.value, flags | (_lib.FLAG_FORCE_SIMT if _FORCE_SIMT else 0),
        ctypes.c_void_p(_lib.stream_handle(dev))), "enable_matmul")
    return out


def _prep_smooth(a, b, smooth_scales):
    """Fuse a / s and b * s into the device quantiser for float32 operands;
    other dtypes are smoothed in their own precision first, as the reference
    does (quant/smoothquant.py:124-126)."""
    if smooth_scales is None:
        return a, b, None
    _check_smoothing(a, b, smooth_scales)
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        a, b = apply_smoothing(a, b, smooth_scales)
        return a, b, None
    s = smooth_scales.to(device=a.device, dtype=torch.float32)
    return a, b, _to_device(s)


def _default_config(config, D, sc_prec):
    if config is None:
        cfg = _DEFAULT_CONFIGS.get((D, sc_prec))
        if cfg is None:
            from .config_helpers import make_sobol_simple_config
            cfg = _DEFAULT_CONFIGS[(D, sc_prec)] = make_sobol_simple_config(D, D, sc_prec)
            _DEFAULT_KEYS[id(cfg)] = (json.dumps(cfg, sort_keys=True), (D, sc_prec))
        return cfg
    return config


@torch.no_grad()
def _sc_matmul_per_tensor(a, b, max_fp_a=None, min_fp_a=None, max_fp_b=None, min_fp_b=None,
                          mode="bipolar", sc_prec=8, config=None, stoc_len=None, rng_levels=None,
                          smooth_scales=None, flags=0):
    """per_tensor path (kernels.py:1053-1226). Without explicit ranges the
    tensors' max/min are reduced on the device (sc_matmul's reference reads them
    back with .item(), matmul.py:227-230); with ``max_fp_a`` / ``min_fp_a``
    (and optionally ``max_fp_b`` / ``min_fp_b``, defaulting to a's, as in
    kernels.py:1092-1095) those host values are used, e.g. global ranges when
    b is sharded over devices."""
    assert a.dim() == b.dim() and a.dim() in (2, 3), f"Expected 2D, got a:{a.dim()}D b:{b.dim()}D"
    assert a.shape[-1] == b.shape[-1], f"Dim mismatch: a={a.shape[-1]}, b={b.shape[-1]}"
    a, b, s = _prep_smooth(a, b, smooth_scales)
    dev_in = a.device
    a, b = _to_device(a), _to_device(b)
    D = a.shape[-1]
    config = _default_config(config, D, sc_prec)
    t = _get_cached_enable_tables(config, sc_prec, a.device, stoc_len, rng_levels)
    ranges = None
    if max_fp_a is not None or min_fp_a is not None:
        if max_fp_a is None or min_fp_a is None:
            raise ValueError("_sc_matmul_per_tensor: give both max_fp_a and min_fp_a")
        mb = max_fp_a if max_fp_b is None else max_fp_b
        nb = min_fp_a if min_fp_b is None else min_fp_b
        ranges = torch.tensor([float(max_fp_a), float(min_fp_a), float(mb), float(nb)],
                              dtype=torch.float64).to(a.device, non_blocking=True)
    y = _launch(_lib.PER_TENSOR, mode, a, b, sc_prec, t, smooth=s, flags=flags, ranges=ranges)
    return y if dev_in.type == "cuda" else _to_host(y)


@torch.no_grad()
def _sc_matmul_per_row(a, b, group_a=1, group_b=1, mode="unipolar", sc_prec=8, config=None,
                       stoc_len=None, rng_levels=None, smooth_scales=None, flags=0):
    """per_row 2D path (kernels.py:1573-1707)."""
    assert a.dim() == 2 and b.dim() == 2, f"Expected 2D, got a:{a.dim()}D b:{b.dim()}D"
    assert a.shape[1] == b.shape[1], f"Inner dim mismatch: {a.shape[1]} vs {b.shape[1]}"
    if mode not in ("bipolar", "unipolar"):
        raise ValueError(f"Unknown mode: {mode}")
    a, b, s = _prep_smooth(a, b, smooth_scales)
    dev_in = a.device
    a, b = _to_device(a), _to_device(b)
    config = _default_config(config, a.shape[1], sc_prec)
    t = _get_cached_enable_tables(config, sc_prec, a.device, stoc_len, rng_levels)
    y = _launch(_lib.PER_ROW, mode, a, b, sc_prec, t, group_a=group_a, group_b=group_b, smooth=s,
                flags=flags)
    return y if dev_in.type == "cuda" else _to_host(y)


@torch.no_grad()
def _sc_matmul_per_row_mlp(a, b, mode="bipolar", sc_prec=8, config=None, group_a=1, group_b=1,
                           chunk_d=0, stoc_len=None, rng_levels=None, smooth_scales=None, flags=0):
    """per_row + chunk_d (kernels.py:1443-1566). With bipolar operands and
    D > chunk_d every chunk is quantised per row on its own and accumulated in
    float32 (kernels.py:1274-1383); group_a / group_b do not apply there, as in
    the reference. Otherwise this is the plain per_row path."""
    assert a.dim() == 2 and b.dim() == 2, f"Expected 2D, got a:{a.dim()}D b:{b.dim()}D"
    assert a.shape[1] == b.shape[1], f"Dim mismatch: a={a.shape[1]}, b={b.shape[1]}"
    D = a.shape[1]
    if not (mode == "bipolar" and chunk_d > 0 and D > chunk_d):
        return _sc_matmul_per_row(a, b, group_a=group_a, group_b=group_b, mode=mode, sc_prec=sc_prec,
                                  config=config, stoc_len=stoc_len, rng_levels=rng_levels,
                                  smooth_scales=smooth_scales, flags=flags)
    a, b, s = _prep_smooth(a, b, smooth_scales)
    dev_in = a.device
    a, b = _to_device(a), _to_device(b)
    config = _default_config(config, chunk_d, sc_prec)
    t = _get_cached_enable_tables(config, sc_prec, a.device, stoc_len, rng_levels)
    y = _launch(_lib.PER_ROW, mode, a, b, sc_prec, t, chunk_d=chunk_d, smooth=s, period=chunk_d,
                flags=flags)
    return y if dev_in.type == "cuda" else _to_host(y)


@torch.no_grad()
def _sc_matmul_per_row_batched(a, b, group_a=1, group_b=1, mode="bipolar", sc_prec=8, config=None,
                               stoc_len=None, rng_levels=None, smooth_scales=None, flags=0):
    """per_row 3D path (kernels.py:1778-1895): (BH, M, D) x (BH, N, D) -> (BH, M, N)."""
    assert a.dim() == 3 and b.dim() == 3, f"Expected 3D, got a:{a.dim()}D b:{b.dim()}D"
    BH, M, D = a.shape
    BH_b, N, D_b = b.shape
    assert BH == BH_b, f"batch mismatch: a BH={BH} vs b BH={BH_b}"
    assert D == D_b, f"inner-dim mismatch: a D={D} vs b D={D_b}"
    if mode not in ("bipolar", "unipolar"):
        raise ValueError(f"Unknown mode: {mode}")
    if mode == "bipolar":
        for G, rows in ((group_a, M), (group_b, N)):
            if not (G == 1 or G >= rows):
                raise NotImplementedError(
                    f"_grouped_symmetric_quant_batched: G={G} not supported (use G=1 or G>=rows)")
    a, b, s = _prep_smooth(a, b, smooth_scales)
    dev_in = a.device
    a, b = _to_device(a), _to_device(b)
    config = _default_config(config, D, sc_prec)
    t = _get_cached_enable_tables(config, sc_prec, a.device, stoc_len, rng_levels)
    y = _launch(_lib.PER_ROW, mode, a, b, sc_prec, t, group_a=group_a, group_b=group_b, smooth=s,
                flags=flags)
    return y if dev_in.type == "cuda" else _to_host(y)


@torch.no_grad()
def _sc_matmul_per_head_bipolar(q_flat, k_flat, sc_prec=8, config=None, stoc_len=None,
                                rng_levels=None, smooth_scales=None, flags=0, **_unused):
    """per_head bipolar path (kernels.py:440-585). Per-head ranges are reduced
    on the device, so the reference's q_maxs / q_mins / k_maxs / k_mins
    arguments are accepted and ignored."""
    if q_flat.dim() != 3 or k_flat.dim() != 3:
        raise ValueError("_sc_matmul_per_head_bipolar: expected 3D (BH, *, D) inputs")
    BH, N, D = q_flat.shape
    BH_k, M, D_k = k_flat.shape
    if BH_k != BH or D_k != D:
        raise ValueError(
            f"_sc_matmul_per_head_bipolar: shape mismatch — q is (BH={BH}, N={N}, D={D}), "
            f"k is (BH={BH_k}, M={M}, D={D_k}); require equal BH and D.")
    a, b, s = _prep_smooth(q_flat, k_flat, smooth_scales)
    dev_in = a.device
    a, b = _to_device(a), _to_device(b)
    config = _default_config(config, D, sc_prec)
    t = _get_cached_enable_tables(config, sc_prec, a.device, stoc_len, rng_levels)
    y = _launch(_lib.PER_HEAD, "bipolar", a, b, sc_prec, t, smooth=s, flags=flags)
    return y if dev_in.type == "cuda" else _to_host(y)


# Re-exports kept for callers that import the quantisers from this module
# (the reference re-exports them at kernels.py:42-52).
from ..quant import (  # noqa: E402,F401
    fused_quantize_bipolar,
    fused_quantize_bipolar_perrow,
    fused_quantize_unipolar,
    fused_quant_bipolar_batched,
    _grouped_symmetric_quant,
    _grouped_asymmetric_quant,
    _grouped_symmetric_quant_batched,
)
