"""Maximal-length LFSR tap search (API of scmp_kernels/sc/lfsr_taps.py).

Taps are lists of bit positions counted from the LSB, highest first, always
including bit ``n_bits - 1``. A tap set is kept when a register seeded with 1
visits all ``2**n_bits - 1`` non-zero states before repeating.

The reference reads its tap lists from a ``lfsr_taps_data.json`` file that it
does not ship (its ``get_default_taps`` raises until the user runs the search);
here :func:`get_taps` falls back to running the search (fast for <= 12 bits)
and caches the result, so ``make_default_config(..., taps=None)`` works.
"""
from __future__ import annotations

import json
from functools import lru_cache
from itertools import combinations
from pathlib import Path
from typing import Optional

from .rng import LFSR

TAPS_FILE = Path(__file__).parent / "lfsr_taps_data.json"


def _is_maximal_length(taps: list[int], n_bits: int, expected_period: int) -> bool:
    lfsr = LFSR(seed=1, length=n_bits, taps=taps)
    seen = set()
    for _ in range(expected_period + 1):
        v = lfsr.step()
        if v in seen:
            return len(seen) == expected_period
        seen.add(v)
    return len(seen) == expected_period


def search_taps(n_bits: int, verbose: bool = False) -> list[list[int]]:
    """All maximal-length tap sets with an even number of taps, in the
    reference's enumeration order (lfsr_taps.py:35-96)."""
    period = 2 ** n_bits - 1
    out = []
    for n_taps in range(2, n_bits + 1, 2):
        for combo in combinations(range(n_bits - 1), n_taps - 1):
            taps = sorted([n_bits - 1] + list(combo), reverse=True)
            if _is_maximal_length(taps, n_bits, period):
                out.append(taps)
    if verbose:
        print(f"Found {len(out)} valid tap configurations for {n_bits} bits")
    return out


def load_taps(filepath: Optional[Path] = None) -> dict[int, list[list[int]]]:
    p = Path(filepath) if filepath is not None else TAPS_FILE
    if not p.exists():
        return {}
    with open(p) as f:
        return {int(k): v for k, v in json.load(f).items()}


def save_taps(taps_dict: dict, filepath: Optional[Path] = None):
    p = Path(filepath) if filepath is not None else TAPS_FILE
    with open(p, "w") as f:
        json.dump({str(k): v for k, v in taps_dict.items()}, f, indent=2)


@lru_cache(maxsize=None)
def _searched(n_bits: int) -> tuple:
    return tuple(tuple(t) for t in search_taps(n_bits))


def get_taps(n_bits: int, filepath: Optional[Path] = None) -> list[list[int]]:
    """Tap sets for ``n_bits``: from the JSON file when present, else searched."""
    stored = load_taps(filepath).get(n_bits)
    if stored:
        return stored
    if n_bits > 16:
        return []
    return [list(t) for t in _searched(n_bits)]
