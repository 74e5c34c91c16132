"""Per-row stream lengths in one call (sc_matmul_levels).

The reference composes mixed precision in its caller (rows classified into
levels, scmp_kernels/mp/config.py:154-191, one sc_matmul per level). Here one
native call must give the same bits: against the reference's own outputs
(the config-4 fixtures, one per level, stacked into one call) and against the
per-level composition on seeded inputs, chunked and not, bipolar and
unipolar, with levels that leave partial tiles and empty levels.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden

from scmp_kernels_b200 import sc_matmul_levels


def test_levels_argument_gates():
    a, b = torch.zeros(4, 16), torch.zeros(5, 16)
    rl = torch.zeros(4, dtype=torch.int32)
    with pytest.raises(ValueError, match="per_row"):
        sc_matmul_levels(a, b, rl, [64], "per_tensor")
    with pytest.raises(ValueError, match="levels"):
        sc_matmul_levels(a, b, rl, [64, 64, 64, 64, 64])
    with pytest.raises(ValueError, match="one level per row"):
        sc_matmul_levels(a, b, rl[:3], [64])
    with pytest.raises(ValueError, match="chunk_d > 0 requires mode='bipolar'"):
        sc_matmul_levels(a, b, rl, [64], mode="unipolar", chunk_d=8)
    with pytest.raises(ValueError, match="rng_levels"):
        sc_matmul_levels(a, b, rl, [64], rng_levels="grid")


gpu = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
DEV = "cuda:0"


def _compose(a, b, rl, Ls, grids, **kw):
    from scmp_kernels_b200 import sc_matmul
    out = torch.empty(a.shape[0], b.shape[0], dtype=torch.float32, device=a.device)
    for lv, (L, G) in enumerate(zip(Ls, grids)):
        rows = torch.nonzero(rl == lv).flatten()
        if rows.numel():
            out[rows] = sc_matmul(a[rows].contiguous(), b, "per_row", stoc_len=L, rng_levels=G, **kw)
    return out


@gpu
@needs_cuda
@pytest.mark.parametrize("grid256", [False, True])
def test_levels_match_reference_fixtures(grid256, env_vars):
    """The config-4 fixtures (the reference's chunked path on rows of each
    tercile, L = 256 / 128 / 64 with rng_levels = L, or the L = 128 rows on
    the 256-level grid) stacked into one call: every row equals the
    reference's output for its level."""
    from scmp_kernels_b200 import _lib
    from scmp_kernels_b200.sc import clear_rng_cache
    env_vars({})
    clear_rng_cache()
    names = ["cfg4_L128_grid256"] if grid256 else ["cfg4_L256", "cfg4_L128", "cfg4_L64"]
    parts = [load_golden(n) for n in names]
    b = parts[0][1]
    for p in parts:
        assert np.array_equal(p[1], b)  # the same rows of b in every fixture
    a = np.concatenate([p[0] for p in parts])
    rl = torch.cat([torch.full((p[0].shape[0],), i, dtype=torch.int32) for i, p in enumerate(parts)])
    Ls = [p[2]["stoc_len"] for p in parts]
    grids = [p[2].get("rng_levels") or 256 for p in parts]
    kw = {k: v for k, v in parts[0][2].items() if k not in ("granularity", "stoc_len", "rng_levels")}
    # rows interleaved across levels, so the permutation is not the identity
    perm = torch.randperm(a.shape[0], generator=torch.Generator().manual_seed(3))
    y = sc_matmul_levels(torch.from_numpy(a)[perm].to(DEV), torch.from_numpy(b).to(DEV), rl[perm].to(DEV), Ls,
                         rng_levels=grids, **kw).cpu().numpy()
    ref = np.concatenate([p[3] for p in parts])[perm.numpy()]
    assert np.array_equal(y, ref)
    assert _lib.device_error() == 0


CASES = [
    # (n, m, d, Ls, rng_levels, kw)
    (700, 300, 320, [256, 128, 64], "stoc_len", dict(mode="bipolar", sc_prec=8, chunk_d=64)),
    (530, 260, 200, [64, 256], None, dict(mode="bipolar", sc_prec=8, chunk_d=64, group_a=4, group_b=4)),
    (300, 520, 640, [256, 64], None, dict(mode="bipolar", sc_prec=8)),
    (270, 300, 384, [64, 64, 64], [64, 48, 32], dict(mode="unipolar", sc_prec=6, group_b=3)),
    (600, 128, 2048, [256, 128], "stoc_len", dict(mode="bipolar", sc_prec=8)),  # long tiles: wide kernel
    (40, 90, 96, [128, 256, 64, 512], None, dict(mode="bipolar", sc_prec=9, chunk_d=32)),
    # short rows (several rows per quantiser block, padding rows among them)
    (330, 70, 120, [64, 256], None, dict(mode="unipolar", sc_prec=8, group_b=3)),
    (270, 300, 64, [256, 128], "stoc_len", dict(mode="bipolar", sc_prec=8)),
]


@gpu
@needs_cuda
@pytest.mark.parametrize("case", range(len(CASES)))
def test_levels_match_per_level_calls(case, env_vars):
    """One call equals the per-level composition bit for bit (row levels from
    a seeded assignment; one case has a level with no rows)."""
    from scmp_kernels_b200 import _lib
    from scmp_kernels_b200.sc import clear_rng_cache
    env_vars({})
    clear_rng_cache()
    n, m, d, Ls, rng, kw = CASES[case]
    g = torch.Generator().manual_seed(500 + case)
    a = (torch.randn(n, d, generator=g) * 2).to(DEV)
    b = (torch.randn(m, d, generator=g) * 0.05).to(DEV)
    nl = len(Ls)
    rl = torch.randint(0, nl, (n,), generator=g, dtype=torch.int32)
    if case == 1:
        rl[rl == 1] = 0  # the second level has no rows
    rl = rl.to(DEV)
    grids = [2 ** kw["sc_prec"] if rng is None else (L if rng == "stoc_len" else rng[i]) for i, L in enumerate(Ls)]
    y = sc_matmul_levels(a, b, rl, Ls, rng_levels=rng, **kw)
    ref = _compose(a, b, rl, Ls, grids, **kw)
    assert torch.equal(y, ref)
    assert _lib.device_error() == 0


@gpu
@needs_cuda
def test_levels_config4_full_size_matches_composition(env_vars):
    """Configuration 4 at full size (12,608 x 3,072 . 768 x 3,072, chunk_d =
    64, rows by range tercile): one call equals the three per-level calls."""
    from scmp_kernels_b200 import _lib, workloads as W
    from scmp_kernels_b200.sc import clear_rng_cache
    env_vars({})
    clear_rng_cache()
    a, b = W.config4(DEV)
    rl, Ls = W.mp_row_level_index(a, 4, (256, 128, 64))
    kw = dict(mode="bipolar", sc_prec=8, chunk_d=64, group_a=4, group_b=4)
    y = sc_matmul_levels(a, b, rl, Ls, rng_levels="stoc_len", **kw)
    ref = _compose(a, b, rl, Ls, Ls, **kw)
    assert torch.equal(y, ref)
    assert _lib.device_error() == 0
