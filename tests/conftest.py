"""Shared test setup: import paths, the `gpu` marker and parity helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "sixi-asi_b200"))
sys.path.insert(0, str(REPO / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def port():
    from oracle import binding

    return binding.port()


@pytest.fixture(scope="session")
def reference():
    from oracle import binding

    r = binding.reference()
    if r is None:
        pytest.skip("reference build (oracle/_ref) not present")
    return r


# Sampled ids must match exactly except where the uniform falls within this distance of a CDF
# boundary of the reference distribution (or the top-p cumulative is this close to top_p).
BOUNDARY_EPS = 1e-6
PROB_RTOL = 1e-5


def near_boundary(oracle, row, params, hist, mask, u) -> bool:
    """True when `u` lies within BOUNDARY_EPS of a CDF boundary of the reference distribution or
    when the top-p decision is within BOUNDARY_EPS of flipping."""
    p = dict(zip(params.dtype.names, params[0]))
    if float(p["temperature"]) <= 0:
        return False
    st, ids, probs, n = oracle.candidates(row, params, hist, mask)
    if st != 0 or n == 0:
        return False
    cdf = np.cumsum(probs)
    if np.any(np.abs(cdf - u) < BOUNDARY_EPS):
        return True
    # top-p boundary: recompute the unrenormalised cumulative with top_p disabled
    q = params.copy()
    q["top_p"] = 1.0
    q["min_p"] = 0.0
    st2, ids2, probs2, n2 = oracle.candidates(row, q, hist, mask)
    tp = float(p["top_p"])
    if 0 < tp < 1 and st2 == 0:
        c2 = np.cumsum(probs2)
        if np.any(np.abs(c2 - tp) < BOUNDARY_EPS):
            return True
    mp = float(p["min_p"])
    if mp > 0 and st2 == 0 and n2 > 0:
        if np.any(np.abs(probs2 / probs2[0] - mp) < 1e-5):
            return True
    return False
