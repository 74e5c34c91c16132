"""Comparator-sequence generators for stochastic computing.

API-compatible with ``scmp_kernels.sc.rng`` (scmp_kernels/sc/rng.py): the same
classes, constructor arguments and ``simulate()`` outputs. The sequences feed
the device-resident enable tables built by :mod:`scmp_kernels_b200.sc.kernels`.
"""
from __future__ import annotations

import random
from abc import ABC, abstractmethod
from typing import Optional

import numpy as np


class RNG(ABC):
    """A generator of ``num_cycles`` integers in ``[0, 2**length)``."""

    @abstractmethod
    def simulate(self, num_cycles: int) -> np.ndarray:
        ...

    @abstractmethod
    def reset(self):
        ...


class LFSR(RNG):
    """Fibonacci shift register (rng.py:32-77).

    Each cycle emits the current register, then shifts it right by one and
    inserts the XOR of the tapped bits (positions counted from the LSB) at bit
    ``length - 1``.
    """

    def __init__(self, seed: int, length: int, taps: list[int]):
        if seed == 0:
            raise ValueError("LFSR seed must be non-zero")
        self.seed = seed
        self.length = length
        self.taps = taps
        self.reg = seed

    def reset(self):
        self.reg = self.seed

    def step(self) -> int:
        out = self.reg
        fb = 0
        for t in self.taps:
            fb ^= (self.reg >> t) & 1
        self.reg = (self.reg >> 1) | (fb << (self.length - 1))
        return out

    def simulate(self, num_cycles: Optional[int] = None) -> np.ndarray:
        n = 2 ** self.length if num_cycles is None else num_cycles
        self.reset()
        return np.fromiter((self.step() for _ in range(n)), dtype=np.int32, count=n)


class TrueRandom(RNG):
    """Python ``random`` draws in ``[0, 2**length - 1]`` (rng.py:80-113).

    The values equal those of the reference, which reseeds the process-wide
    ``random`` module; this class draws from a private ``random.Random(seed)``
    instead, so simulating it leaves the caller's global random state alone.
    """

    def __init__(self, seed: int, length: int):
        self.seed = seed
        self.length = length
        self.max_val = 2 ** length - 1
        self._r = random.Random(seed)

    def reset(self):
        self._r = random.Random(self.seed)

    def simulate(self, num_cycles: Optional[int] = None) -> np.ndarray:
        n = 2 ** self.length if num_cycles is None else num_cycles
        self.reset()
        return np.array([self._r.randint(0, self.max_val) for _ in range(n)], dtype=np.int32)


class Sobol(RNG):
    """Gray-code Sobol sequence with SCGen direction numbers (rng.py:116-239).

    Direction vector ``i`` is ``int(seed[i] / 2**(i+1) * 2**length)``; step
    ``idx`` emits the running value and then XORs in the direction vector of
    the lowest zero bit of ``idx``. The default Q seed is all ones; the default
    K seed decorrelates K from Q.
    """

    def __init__(self, length: int, seed: Optional[list] = None, seed_type: str = "q"):
        self.length = length
        self.max_val = 2 ** length
        self.seed = list(seed) if seed is not None else self._default_seed(seed_type)
        self._direction_vectors = self._compute_direction_vectors()
        self._index = 0
        self._value = 0

    def _default_seed(self, seed_type: str) -> list:
        if seed_type == "k":
            if self.length == 8:
                return [1, 1, 1, 1, 9, 1, 41, 255]
            s = [1] * self.length
            if self.length >= 5:
                s[4] = 9
            if self.length >= 7:
                s[6] = 41
            return s
        return [1] * self.length

    def _compute_direction_vectors(self) -> list:
        return [int(self.seed[i] / (1 << (i + 1)) * (1 << self.length)) for i in range(self.length)]

    @staticmethod
    def _lsz(n: int) -> int:
        pos = 0
        while (n >> pos) & 1:
            pos += 1
        return pos

    def reset(self):
        self._index = 0
        self._value = 0

    def _step(self) -> int:
        val = self._value
        k = self._lsz(self._index)
        self._index += 1
        if k < self.length:
            self._value ^= self._direction_vectors[k]
        return val

    def step(self) -> int:
        return self._step()

    def simulate(self, num_cycles: Optional[int] = None) -> np.ndarray:
        n = 2 ** self.length if num_cycles is None else num_cycles
        self.reset()
        return np.fromiter((self._step() for _ in range(n)), dtype=np.int32, count=n)

    @staticmethod
    def random_seed(length: int) -> list:
        """A valid random seed: s0 = 1, s_i odd in [1, 2**(i+1))."""
        return [1] + [random.randint(0, (1 << (i + 1)) // 2 - 1) * 2 + 1 for i in range(1, length)]


def create_rng(rng_type: str, length: int, **kwargs) -> RNG:
    """Factory used by the RNG pool (rng.py:242-268)."""
    if rng_type == "lfsr":
        return LFSR(seed=kwargs["seed"], length=length, taps=kwargs["taps"])
    if rng_type == "true_random":
        return TrueRandom(seed=kwargs["seed"], length=length)
    if rng_type == "sobol":
        return Sobol(length=length, seed=kwargs.get("seed"), seed_type=kwargs.get("seed_type", "q"))
    raise ValueError(f"Unknown RNG type: {rng_type}")
