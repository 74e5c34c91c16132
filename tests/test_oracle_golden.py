"""The CPU oracle against golden vectors produced by the reference itself
(tests/golden/gen_golden.py runs the reference's sc_matmul under
TRITON_INTERPRET=1). Every comparison is bit-exact."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_names, load_golden
from oracle import sc_oracle as O


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference(name):
    a, b, p, out, s, env = load_golden(name)
    e = {k: v for k, v in os.environ.items() if not k.startswith("SC_")}
    e.update(env)
    g = p.pop("granularity")
    y = O.sc_matmul(a, b, g, smooth_scales=s, env=e, **p)
    assert y.shape == out.shape
    assert np.array_equal(y, out), f"max |diff| {np.abs(y - out).max()}"


RNG = np.load(os.path.join(GOLDEN, "rng_golden.npz"))


@pytest.mark.parametrize("p", [4, 6, 8])
def test_sobol_sequences(p):
    assert np.array_equal(O.sobol_sequence(p, seed_type="q"), RNG[f"sobol_q_p{p}"])
    assert np.array_equal(O.sobol_sequence(p, seed_type="k"), RNG[f"sobol_k_p{p}"])


def test_lfsr_sequences_and_taps():
    assert np.array_equal(O.lfsr_sequence(125, 8, [7, 2, 1, 0]), RNG["lfsr_p8_s125"])
    assert np.array_equal(O.lfsr_sequence(21, 6, [5, 0]), RNG["lfsr_p6_s21"])
    cfg = {"rng_pool": [{"type": "lfsr", "seed": 125, "taps": [7, 2, 1, 0]}],
           "sng": {"q": [{"rng_id": 0, "scramble": None}] * 5,
                   "k": [{"rng_id": 0, "scramble": list(range(7, -1, -1))}] * 5}}
    assert np.array_equal(O.bank_sequences(cfg, 8, "q"), RNG["bank_default_q"])
    assert np.array_equal(O.bank_sequences(cfg, 8, "k"), RNG["bank_default_k"])


PREP = [(256, 256), (64, 256), (64, 64), (100, 128), (256, 300), (40, 100)]


@pytest.mark.parametrize("L,G", PREP)
@pytest.mark.parametrize("mode", ["bitrev", "counter", "off"])
def test_prepare_prefix(L, G, mode):
    cfg = O.make_sobol_simple_config(6, 6, 8)
    rb = O.bank_sequences(cfg, 8, "k")
    got = O.prepare_rng_prefix(rb, 8, L, G, env={"SC_OWEN_MODE": mode})
    assert np.array_equal(got, RNG[f"prep_L{L}_G{G}_{mode}"])


@pytest.mark.parametrize("L,G", PREP)
def test_tables(L, G):
    cfg = O.make_sobol_simple_config(6, 6, 8)
    T = O.Tables(cfg, 8, L, G, env={})
    assert np.array_equal(T.kt, RNG[f"ktab_L{L}_G{G}"])
    cum = RNG[f"cum_L{L}_G{G}"]
    for d in range(6):
        assert np.array_equal(O.count_table(T.rb[d], L, T.V), cum[d])
