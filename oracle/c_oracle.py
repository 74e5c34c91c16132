"""Multi-threaded CPU oracle -- TEST INFRASTRUCTURE ONLY.

``sc_oracle`` (numpy) with its integer accumulator computed by the OpenMP C
restatement in sc_enable_sum.c. Used as the CPU baseline of bench.py and for
parity cases too large for the numpy loop; never by the product path.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import sc_oracle as O

_lib = None


def _load():
    global _lib
    if _lib is None:
        from .build import OUT, build
        if not os.path.exists(OUT):
            build()
        lib = ctypes.CDLL(OUT)
        lib.sc_enable_sum.restype = None
        _lib = lib
    return _lib


def available() -> bool:
    try:
        _load()
        return True
    except Exception:
        return False


def enable_sum_c(kt, rb, L, ba, bb, sa=None, sb=None, threads=0):
    """Same contract as sc_oracle.enable_sum."""
    N, D = ba.shape
    M = bb.shape[0]
    V = kt.shape[1]
    rows, rowmap = np.unique(rb[:, :L], axis=0, return_inverse=True)
    cum = np.ascontiguousarray(np.stack([O.count_table(r, L, V) for r in rows]), dtype=np.int32)
    kk = np.ascontiguousarray(kt[np.arange(D)[None, :], ba.astype(np.int64)], dtype=np.int32)
    bbi = np.ascontiguousarray(bb, dtype=np.int32)
    rm = np.ascontiguousarray(rowmap.reshape(-1), dtype=np.int32)
    S = np.zeros((N, M), dtype=np.int64)
    P = ctypes.c_void_p
    sa_p = P(np.ascontiguousarray(sa, dtype=np.int8).ctypes.data) if sa is not None else None
    sb_p = P(np.ascontiguousarray(sb, dtype=np.int8).ctypes.data) if sb is not None else None
    keep = (sa if sa is None else np.ascontiguousarray(sa, dtype=np.int8),
            sb if sb is None else np.ascontiguousarray(sb, dtype=np.int8))
    if sa is not None:
        sa_p, sb_p = P(keep[0].ctypes.data), P(keep[1].ctypes.data)
    _load().sc_enable_sum(ctypes.c_int(N), ctypes.c_int(M), ctypes.c_int(D), P(kk.ctypes.data),
                          P(bbi.ctypes.data), sa_p, sb_p, P(cum.ctypes.data), P(rm.ctypes.data),
                          ctypes.c_int(L + 1), ctypes.c_int(V), P(S.ctypes.data), ctypes.c_int(threads))
    return S


def sc_matmul(a, b, granularity="per_row", threads=0, env=None, **kw):
    """sc_oracle.sc_matmul with the C accumulator."""
    old = O.enable_sum
    O.enable_sum = lambda kt, rb, L, ba, bb, sa=None, sb=None: enable_sum_c(kt, rb, L, ba, bb, sa, sb, threads)
    try:
        return O.sc_matmul(a, b, granularity, env={} if env is None else env, **kw)
    finally:
        O.enable_sum = old
