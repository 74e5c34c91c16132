"""Shared test setup: the `gpu` marker, fixture loading, repo on sys.path."""
from __future__ import annotations

import glob
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def golden_names():
    return sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if not f.endswith("rng_golden.npz"))


def load_golden(name):
    """(a, b, params, out, smooth_scales or None, env) of one fixture."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    p = json.loads(str(z["params"]))
    env = p.pop("env", {})
    s = z["smooth_scales"] if "smooth_scales" in z else None
    return z["a"], z["b"], p, z["out"], s, env


@pytest.fixture
def env_vars(monkeypatch):
    def apply(env):
        for k in ("SC_OWEN_MODE", "SC_DISABLE_OWEN", "SC_SCRAMBLE_RESCALE"):
            monkeypatch.delenv(k, raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
    return apply
