"""Host-side logic of the package, on CPU: RNG sequences, prefix / Owen /
rescale preparation and config builders against the reference's own outputs."""
from __future__ import annotations

import os
import random

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from scmp_kernels_b200.sc import config_helpers as C
from scmp_kernels_b200.sc import kernels as K
from scmp_kernels_b200.sc.lfsr_taps import search_taps
from scmp_kernels_b200.sc.rng import LFSR, Sobol, TrueRandom, create_rng
from scmp_kernels_b200.sc.sng import RNGPool, SNGBank

RNG = np.load(os.path.join(GOLDEN, "rng_golden.npz"))


@pytest.mark.parametrize("p", [4, 6, 8])
def test_sobol(p):
    assert np.array_equal(Sobol(p, seed_type="q").simulate(), RNG[f"sobol_q_p{p}"])
    assert np.array_equal(Sobol(p, seed_type="k").simulate(), RNG[f"sobol_k_p{p}"])


def test_lfsr_and_taps():
    assert np.array_equal(LFSR(125, 8, [7, 2, 1, 0]).simulate(), RNG["lfsr_p8_s125"])
    assert np.array_equal(LFSR(21, 6, [5, 0]).simulate(), RNG["lfsr_p6_s21"])
    for p in (4, 6, 8):
        assert search_taps(p)[0] == list(RNG[f"taps_p{p}"])
    with pytest.raises(ValueError):
        LFSR(0, 8, [7, 2, 1, 0])
    with pytest.raises(ValueError):
        create_rng("xorshift", 8)


def test_truerandom_leaves_global_state():
    random.seed(5)
    x = random.random()
    random.seed(5)
    s1 = TrueRandom(7, 8).simulate()
    assert random.random() == x
    r = random.Random(7)
    assert list(s1) == [r.randint(0, 255) for _ in range(256)]


def test_default_config_bank():
    cfg = C.make_default_config(5, 5, 8, taps=[7, 2, 1, 0], seed=125)
    pool = RNGPool(cfg["rng_pool"], 8)
    assert np.array_equal(SNGBank(pool, cfg["sng"]["q"]).get_all_sequences(256), RNG["bank_default_q"])
    assert np.array_equal(SNGBank(pool, cfg["sng"]["k"]).get_all_sequences(256), RNG["bank_default_k"])
    assert C.make_default_config(2, 2, 8)["rng_pool"][0]["taps"] == [7, 2, 1, 0]


PREP = [(256, 256), (64, 256), (64, 64), (100, 128), (256, 300), (40, 100)]


@pytest.mark.parametrize("L,G", PREP)
@pytest.mark.parametrize("mode", ["bitrev", "counter", "off"])
def test_prepare_prefix(L, G, mode, monkeypatch):
    monkeypatch.setenv("SC_OWEN_MODE", mode)
    cfg = C.make_sobol_simple_config(6, 6, 8)
    _, rb = K._get_cached_sequences(cfg, 8, "cpu")
    assert np.array_equal(K._prepare_rng_prefix(rb, 8, L, G), RNG[f"prep_L{L}_G{G}_{mode}"])


def _emulate_tables(ra, rb, L, lp, vcap):
    """numpy restatement of the device table kernels (csrc/tables.cu)."""
    v = np.arange(vcap + 1)
    ktab = (ra[:, :L, None] < v).sum(axis=1)
    bits = (rb[:, :L, None] < v)                        # (rows, L, V)
    bits = np.pad(bits, ((0, 0), (0, lp - L), (0, 0)))
    w = bits.reshape(rb.shape[0], lp // 32, 32, vcap + 1)
    pat = (w.astype(np.uint64) << np.arange(32, dtype=np.uint64)[None, None, :, None]).sum(axis=2)
    return ktab, pat.transpose(0, 2, 1).astype(np.uint32)


@pytest.mark.parametrize("L,G", PREP)
def test_table_encoding_reproduces_cum_indicator(L, G):
    """popcount of the first k bits of pattern[v] is the reference's cum[k][v];
    ktab equals the reference's k_table on [0, G]."""
    cfg = C.make_sobol_simple_config(6, 6, 8)
    qa, kb = K._get_cached_sequences(cfg, 8, "cpu")
    ra = K._prepare_rng_prefix(qa, 8, L, G)
    rb = K._prepare_rng_prefix(kb, 8, L, G)
    vcap = max(G, int(max(ra.max(), rb.max())) + 1)
    lp = max(32, K._next_pow2(L))
    ktab, pat = _emulate_tables(ra, rb, L, lp, vcap)
    ref_k = RNG[f"ktab_L{L}_G{G}"]
    assert np.array_equal(ktab[:, :G + 1], ref_k[:, :G + 1])
    cum = RNG[f"cum_L{L}_G{G}"]
    V = cum.shape[2]
    for d in range(6):
        for k in range(0, L + 1, max(1, L // 16)):
            words = pat[d, :, :]                          # (vcap+1, lp/32)
            full, rem = divmod(k, 32)
            c = np.zeros(vcap + 1, dtype=np.int64)
            for w in range(full):
                c += np.array([bin(int(x)).count("1") for x in words[:, w]])
            if rem:
                c += np.array([bin(int(x) & ((1 << rem) - 1)).count("1") for x in words[:, full]])
            vv = min(V, vcap + 1)
            assert np.array_equal(c[:vv], cum[d, k, :vv])


def test_dedup_single_row_for_default_sobol():
    cfg = C.make_sobol_simple_config(4096, 4096, 8)
    qa, kb = K._get_cached_sequences(cfg, 8, "cpu")
    for L, G in ((256, 256), (128, 128), (64, 256)):
        os.environ.pop("SC_OWEN_MODE", None)
        ra = K._prepare_rng_prefix(qa, 8, L, G)
        ua = np.unique(ra, axis=0)
        # full-length default Sobol: one distinct row; Owen-scrambled prefixes:
        # at most 2**p distinct masks
        if L == 256 and G == 256:
            assert ua.shape[0] == 1
        else:
            assert 1 < ua.shape[0] <= 256


def test_config_builders_seeded_like_reference():
    random.seed(1234)
    cfg = C.make_per_element_scramble_config(24, 24, 8, taps=[7, 2, 1, 0], seed=99)
    import json
    z = np.load(os.path.join(GOLDEN, "e_lfsr_perelem.npz"))
    assert json.loads(str(z["params"]))["config"] == cfg


@pytest.mark.parametrize("name,build", [
    ("e_cfg_antithetic", lambda: C.make_sobol_antithetic_config(40, 40, 8)),
    ("e_cfg_altseed8", lambda: C.make_sobol_altseed_config(40, 40, 8)),
    ("e_cfg_altseed6_prefix", lambda: C.make_sobol_altseed_config(36, 36, 6)),
    ("e_cfg_custom_seed", lambda: (random.seed(77), C.make_sobol_custom_seed_config(
        32, 32, 8, q_seed=[1, 1, 3, 5, 15, 17, 51, 85], k_seed=[1, 3, 7, 1, 9, 33, 41, 255],
        use_scrambling=True))[1]),
    ("e_cfg_dse", lambda: (random.seed(2024), C.make_sobol_dse_config(32, 32, 8))[1]),
])
def test_sobol_config_builders_match_fixture_configs(name, build):
    """The Sobol builders (config_helpers.py:610-763) give the configs the
    fixtures were generated with: the reference's own builders for the
    antithetic, alternative-seed and custom-seed variants (same draws from
    Python's ``random`` for the scrambles), this package's for DSE, whose
    reference builder cannot be imported."""
    import json
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    assert json.loads(str(z["params"]))["config"] == build()


@pytest.mark.parametrize("n,L,g", [(4096, 256, 1), (8192, 64, 1), (1101, 256, 5), (1101, 64, 3),
                                   (1024, 32, 1), (12608, 256, 4), (2000, 128, 7), (1024, 512, 1)])
def test_host_pipeline_row_blocks(n, L, g):
    """a's blocks on the streamed host path: they tile [0, n) in order, inner
    boundaries fall on whole row groups, the first block is 2^18 / L rows in
    whole 256-row tiles, between a quarter and half of a (config 2: a quarter;
    config 5, L = 64: half)."""
    from scmp_kernels_b200.sc.matmul import _a_blocks
    bl = _a_blocks(n, L, g)
    assert bl[0][0] == 0 and bl[-1][1] == n
    assert all(x[1] == y[0] and x[0] < x[1] for x, y in zip(bl, bl[1:]))
    assert all(x[1] % g == 0 for x in bl[:-1])
    first = bl[0][1]
    assert (n + 3) // 4 <= first <= (n + 1) // 2 + g
    if (n, L) == (4096, 256):
        assert bl == [(0, 1024), (1024, 3072), (3072, 4096)]
    if (n, L) == (8192, 64):
        assert first == 4096
