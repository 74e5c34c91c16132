"""Stochastic number generators: an RNG pool plus per-element bit scrambles.

API-compatible with ``scmp_kernels.sc.sng`` (scmp_kernels/sc/sng.py).
"""
from __future__ import annotations

import random
from typing import Optional

import numpy as np

from .rng import RNG, create_rng


def apply_scramble(sequence: np.ndarray, scramble: list[int]) -> np.ndarray:
    """Bit permutation: output bit ``i`` takes source bit ``scramble[i]`` (sng.py:15-29)."""
    out = np.zeros_like(sequence)
    for i, src in enumerate(scramble):
        out |= ((sequence >> src) & 1) << i
    return out


def apply_scramble_batch(sequences: np.ndarray, scrambles: list, sc_prec: int) -> np.ndarray:
    """Row-wise :func:`apply_scramble`; a ``None`` scramble keeps its row (sng.py:32-53)."""
    out = np.zeros_like(sequences)
    for bit in range(sc_prec):
        src = np.array([s[bit] if s is not None else bit for s in scrambles])
        out |= ((sequences >> src[:, None]) & 1) << bit
    return out


def reverse_permutation(n_bits: int) -> list[int]:
    """The bit-reversal scramble (sng.py:56-58)."""
    return list(range(n_bits - 1, -1, -1))


def generate_random_permutation(n_bits: int) -> list[int]:
    """A shuffle of the bit positions drawn from the process-wide ``random``
    module, as in the reference (sng.py:61-66), so seeded config builders
    reproduce its configs."""
    perm = list(range(n_bits))
    random.shuffle(perm)
    return perm


class RNGPool:
    """Pool of RNGs built from config dicts; sequences are cached per RNG id
    (sng.py:69-120)."""

    def __init__(self, rng_configs: list[dict], sc_prec: int):
        self.sc_prec = sc_prec
        self.rngs: list[RNG] = [
            create_rng(rng_type=c.get("type", "lfsr"), length=sc_prec,
                       **{k: v for k, v in c.items() if k != "type"})
            for c in rng_configs
        ]
        self._sequence_cache: dict[int, np.ndarray] = {}

    def __len__(self):
        return len(self.rngs)

    def get_sequence(self, rng_id: int, stoc_len: int) -> np.ndarray:
        if rng_id not in self._sequence_cache:
            self._sequence_cache[rng_id] = self.rngs[rng_id].simulate(stoc_len)
        return self._sequence_cache[rng_id]

    def clear_cache(self):
        self._sequence_cache.clear()


class SNG:
    """One element's generator: a pool RNG and an optional scramble (sng.py:123-157)."""

    def __init__(self, rng_pool: RNGPool, rng_id: int, scramble: Optional[list[int]] = None):
        self.rng_pool = rng_pool
        self.rng_id = rng_id
        self.scramble = scramble

    def get_sequence(self, stoc_len: int) -> np.ndarray:
        seq = self.rng_pool.get_sequence(self.rng_id, stoc_len)
        return apply_scramble(seq, self.scramble) if self.scramble is not None else seq.copy()


class SNGBank:
    """The generators of one operand's elements (sng.py:160-230)."""

    def __init__(self, rng_pool: RNGPool, sng_configs: list[dict]):
        self.rng_pool = rng_pool
        self.sng_configs = sng_configs
        self.sngs = [SNG(rng_pool, c["rng_id"], c.get("scramble")) for c in sng_configs]

    def __len__(self):
        return len(self.sngs)

    def get_all_sequences(self, stoc_len: int) -> np.ndarray:
        """``(n_elements, stoc_len)`` int32 sequences."""
        n = len(self.sngs)
        ids = {s.rng_id for s in self.sngs}
        if len(ids) == 1:
            base = self.rng_pool.get_sequence(next(iter(ids)), stoc_len)
            scr = [s.scramble for s in self.sngs]
            rows = np.broadcast_to(base, (n, stoc_len)).copy()
            if all(s is None for s in scr):
                return rows
            return apply_scramble_batch(rows, scr, self.rng_pool.sc_prec)
        out = np.zeros((n, stoc_len), dtype=np.int32)
        for i, s in enumerate(self.sngs):
            out[i] = s.get_sequence(stoc_len)
        return out
