"""Builders of RNG/SNG config dicts (API of scmp_kernels/sc/config_helpers.py).

A config names an RNG pool (``rng_pool``: LFSR / Sobol / true-random entries)
and, per element of each operand, which pool RNG it draws from and an optional
bit scramble (``sng.q`` for operand a, ``sng.k`` for operand b). ``sc_matmul``
uses ``make_sobol_simple_config`` when ``config=None``.

Builders that draw random taps, seeds or scrambles use the process-wide
``random`` module like the reference, so a seeded caller gets the same config.
"""
from __future__ import annotations

import random
from typing import Optional

from .lfsr_taps import get_taps
from .rng import Sobol
from .sng import generate_random_permutation, reverse_permutation


def get_taps_choices(sc_prec: int) -> list[list[int]]:
    taps = get_taps(sc_prec)
    if not taps:
        raise ValueError(f"No pre-computed taps for sc_prec={sc_prec}. "
                         f"Run `python lfsr_taps.py {sc_prec}` to generate.")
    return taps


def get_default_taps(sc_prec: int) -> list[int]:
    return get_taps_choices(sc_prec)[0]


def _cfg(pool, q, k):
    return {"rng_pool": pool, "sng": {"q": q, "k": k}}


def make_default_config(q_e: int, k_e: int, sc_prec: int, taps: Optional[list[int]] = None,
                        seed: int = 125) -> dict:
    """One shared LFSR; every K element bit-reversed (config_helpers.py:51-82)."""
    taps = get_default_taps(sc_prec) if taps is None else taps
    ks = reverse_permutation(sc_prec)
    return _cfg([{"type": "lfsr", "seed": seed, "taps": taps}],
                [{"rng_id": 0, "scramble": None} for _ in range(q_e)],
                [{"rng_id": 0, "scramble": ks} for _ in range(k_e)])


def make_independent_config(q_e: int, k_e: int, sc_prec: int, q_taps: list[int], k_taps: list[int],
                            q_seed: int, k_seed: int, q_scramble: Optional[list[int]] = None,
                            k_scramble: Optional[list[int]] = None) -> dict:
    """Separate LFSRs for Q and K (config_helpers.py:85-116)."""
    return _cfg([{"type": "lfsr", "seed": q_seed, "taps": q_taps},
                 {"type": "lfsr", "seed": k_seed, "taps": k_taps}],
                [{"rng_id": 0, "scramble": q_scramble} for _ in range(q_e)],
                [{"rng_id": 1, "scramble": k_scramble} for _ in range(k_e)])


def make_per_element_scramble_config(q_e: int, k_e: int, sc_prec: int,
                                     taps: Optional[list[int]] = None, seed: int = 125,
                                     k_reverse_of_q: bool = True) -> dict:
    """One LFSR; each element its own random scramble (config_helpers.py:119-163)."""
    taps = get_default_taps(sc_prec) if taps is None else taps
    assert q_e == k_e, "Q and K must have same embedding size for paired scrambling"
    q, k = [], []
    for _ in range(q_e):
        sq = generate_random_permutation(sc_prec)
        sk = list(reversed(sq)) if k_reverse_of_q else generate_random_permutation(sc_prec)
        q.append({"rng_id": 0, "scramble": sq})
        k.append({"rng_id": 0, "scramble": sk})
    return _cfg([{"type": "lfsr", "seed": seed, "taps": taps}], q, k)


def make_fully_independent_config(q_e: int, k_e: int, sc_prec: int,
                                  taps_choices: Optional[list[list[int]]] = None) -> dict:
    """A random LFSR per element (config_helpers.py:166-209)."""
    taps_choices = get_taps_choices(sc_prec) if taps_choices is None else taps_choices
    pool, qi, ki = [], [], []
    for ids, n in ((qi, q_e), (ki, k_e)):
        for _ in range(n):
            pool.append({"type": "lfsr", "seed": None, "taps": random.choice(taps_choices)})
            pool[-1]["seed"] = random.randint(1, 2 ** sc_prec - 1)
            ids.append(len(pool) - 1)
    return _cfg(pool, [{"rng_id": i, "scramble": None} for i in qi],
                [{"rng_id": i, "scramble": None} for i in ki])


def make_separated_random_config(q_e: int, k_e: int, sc_prec: int,
                                 taps_choices: Optional[list[list[int]]] = None) -> dict:
    """Random taps and seeds; Q on RNG 0, K on RNG 1 (config_helpers.py:212-245)."""
    taps_choices = get_taps_choices(sc_prec) if taps_choices is None else taps_choices
    qt, kt = random.choice(taps_choices), random.choice(taps_choices)
    qs, ks = random.randint(1, 2 ** sc_prec - 1), random.randint(1, 2 ** sc_prec - 1)
    return _cfg([{"type": "lfsr", "seed": qs, "taps": qt}, {"type": "lfsr", "seed": ks, "taps": kt}],
                [{"rng_id": 0, "scramble": None} for _ in range(q_e)],
                [{"rng_id": 1, "scramble": None} for _ in range(k_e)])


def make_random_config(q_e: int, k_e: int, sc_prec: int,
                       taps_choices: Optional[list[list[int]]] = None,
                       use_scrambling: bool = True) -> dict:
    """Random LFSR pair plus random per-element scrambles (config_helpers.py:248-299)."""
    taps_choices = get_taps_choices(sc_prec) if taps_choices is None else taps_choices
    qt, kt = random.choice(taps_choices), random.choice(taps_choices)
    qs, ks = random.randint(1, 2 ** sc_prec - 1), random.randint(1, 2 ** sc_prec - 1)
    q = [{"rng_id": 0, "scramble": generate_random_permutation(sc_prec)
          if use_scrambling and random.random() > 0.5 else None} for _ in range(q_e)]
    k = [{"rng_id": 1, "scramble": generate_random_permutation(sc_prec)
          if use_scrambling and random.random() > 0.5 else None} for _ in range(k_e)]
    return _cfg([{"type": "lfsr", "seed": qs, "taps": qt}, {"type": "lfsr", "seed": ks, "taps": kt}], q, k)


def make_single_rng_reverse_config(q_e: int, k_e: int, sc_prec: int,
                                   taps_choices: Optional[list[list[int]]] = None,
                                   use_per_element_scrambling: bool = True) -> dict:
    """One random LFSR; K scrambles are the reverse of Q's (config_helpers.py:302-355)."""
    taps_choices = get_taps_choices(sc_prec) if taps_choices is None else taps_choices
    assert q_e == k_e, "Q and K must have same size for paired reverse scrambling"
    taps = random.choice(taps_choices)
    seed = random.randint(1, 2 ** sc_prec - 1)
    q, k = [], []
    if use_per_element_scrambling:
        for _ in range(q_e):
            sq = generate_random_permutation(sc_prec)
            q.append({"rng_id": 0, "scramble": sq})
            k.append({"rng_id": 0, "scramble": list(reversed(sq))})
    else:
        ks = reverse_permutation(sc_prec)
        q = [{"rng_id": 0, "scramble": None} for _ in range(q_e)]
        k = [{"rng_id": 0, "scramble": ks} for _ in range(q_e)]
    return _cfg([{"type": "lfsr", "seed": seed, "taps": taps}], q, k)


def make_sobol_simple_config(q_e: int, k_e: int, sc_prec: int = 8) -> dict:
    """Default Sobol config: Q seed all ones, K the decorrelated seed
    (config_helpers.py:583-607)."""
    return _cfg([{"type": "sobol", "seed_type": "q"}, {"type": "sobol", "seed_type": "k"}],
                [{"rng_id": 0, "scramble": None} for _ in range(q_e)],
                [{"rng_id": 1, "scramble": None} for _ in range(k_e)])


def make_sobol_antithetic_config(q_e: int, k_e: int, sc_prec: int = 8) -> dict:
    """Sobol pair with a ``complement`` flag on K (config_helpers.py:610-634).
    As in the reference, the stream generators ignore the flag."""
    return _cfg([{"type": "sobol", "seed_type": "q"}, {"type": "sobol", "seed_type": "k"}],
                [{"rng_id": 0, "scramble": None} for _ in range(q_e)],
                [{"rng_id": 1, "scramble": None, "complement": True} for _ in range(k_e)])


def make_sobol_altseed_config(q_e: int, k_e: int, sc_prec: int = 8,
                              k_seed: Optional[list[int]] = None) -> dict:
    """Sobol Q with an alternative K direction seed (config_helpers.py:637-672)."""
    if k_seed is None:
        k_seed = ([1, 3, 7, 15, 31, 63, 127, 255] if sc_prec == 8
                  else [(1 << (i + 1)) - 1 for i in range(sc_prec)])
    return _cfg([{"type": "sobol", "seed_type": "q"}, {"type": "sobol", "seed": list(k_seed)}],
                [{"rng_id": 0, "scramble": None} for _ in range(q_e)],
                [{"rng_id": 1, "scramble": None} for _ in range(k_e)])


def make_sobol_dse_config(q_e: int, k_e: int, sc_prec: int, use_scrambling: bool = True) -> dict:
    """Random valid Sobol seeds plus optional random scrambles
    (config_helpers.py:675-721; the reference's ``from rng import Sobol`` import
    fails, this builder imports the class correctly)."""
    qs, ks = Sobol.random_seed(sc_prec), Sobol.random_seed(sc_prec)
    q = [{"rng_id": 0, "scramble": generate_random_permutation(sc_prec)
          if use_scrambling and random.random() > 0.5 else None} for _ in range(q_e)]
    k = [{"rng_id": 1, "scramble": generate_random_permutation(sc_prec)
          if use_scrambling and random.random() > 0.5 else None} for _ in range(k_e)]
    return _cfg([{"type": "sobol", "seed": qs}, {"type": "sobol", "seed": ks}], q, k)


def make_sobol_custom_seed_config(q_e: int, k_e: int, sc_prec: int, q_seed: list = None,
                                  k_seed: list = None, use_scrambling: bool = False) -> dict:
    """Sobol pair with caller-given seeds (config_helpers.py:724-763)."""
    q = [{"rng_id": 0, "scramble": generate_random_permutation(sc_prec) if use_scrambling else None}
         for _ in range(q_e)]
    k = [{"rng_id": 1, "scramble": generate_random_permutation(sc_prec) if use_scrambling else None}
         for _ in range(k_e)]
    return _cfg([{"type": "sobol", "seed": q_seed, "seed_type": "q"},
                 {"type": "sobol", "seed": k_seed, "seed_type": "k"}], q, k)
