"""The C-ABI library loads and exports every function include/scmp_b200.h
declares; argument validation answers without touching a GPU."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import REPO
from scmp_kernels_b200 import _lib

HEADER = os.path.join(REPO, "include", "scmp_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(scmp_[a-z0-9_]+)\s*\(", src)))


def test_library_builds_and_loads():
    from scmp_kernels_b200 import build
    build.build()
    assert _lib.load().scmp_abi_version() == _lib.ABI_VERSION == 4


def test_every_declared_symbol_is_exported():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_invalid_arguments_are_rejected_without_gpu():
    lib = _lib.load()
    d = _lib.MatmulDesc(granularity=7, mode=0, sc_prec=8, stoc_len=256, rng_levels=256, lp=256,
                        vcap=256, batch=1, n=4, m=4, d=8, group_a=1, group_b=1)
    size = ctypes.c_size_t()
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_INVALID_ARG
    assert b"granularity" in lib.scmp_last_error()
    d.granularity = _lib.PER_ROW
    d.lp = 100
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_INVALID_ARG
    d.lp = 256
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_OK
    assert size.value >= 2 * (4 * 8 + 4 * 8)
    d.n_out_peers = _lib.MAX_OUT_PEERS + 1
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_INVALID_ARG
    d.n_out_peers, d.out_ld = 2, 3  # destinations narrower than m
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_INVALID_ARG
    assert b"out_ld" in lib.scmp_last_error()
    d.n_out_peers, d.out_ld = 0, 0
    d.batch, d.group_a = 2, 3
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.SCMP_ERR_UNSUPPORTED)
    # b already quantised in the workspace: per_row without chunking only
    d.batch, d.group_a = 1, 1
    d.flags = _lib.FLAG_B_READY
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_OK
    d.granularity = _lib.PER_TENSOR
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_INVALID_ARG
    assert b"B_READY" in lib.scmp_last_error()
    d.granularity, d.chunk_d, d.d = _lib.PER_ROW, 4, 8
    assert lib.scmp_sc_matmul_workspace_size(ctypes.byref(d), ctypes.byref(size)) == _lib.SCMP_ERR_INVALID_ARG
    d.flags, d.chunk_d = 0, 0
    assert lib.scmp_build_tables(None, 1, None, 1, 0, 32, 8, None, None, None, None) == _lib.SCMP_ERR_INVALID_ARG
    with pytest.raises(ValueError):
        _lib.check(_lib.SCMP_ERR_INVALID_ARG)
