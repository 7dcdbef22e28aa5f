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


# Every mismatch a parity test excused (rows within BOUNDARY_EPS of a decision boundary), with the
# kind of boundary and its distance; summarised at the end of the session.
EXCUSED: list[dict] = []
COMPARED = {"rows": 0}


def max_excused(n_rows: int) -> int:
    """Excused mismatches a parity check accepts over n_rows sampled rows: 1 per 256 rows (at least
    1). With uniforms drawn independently of the rows, a uniform lands within 1e-6 of one of a few
    hundred CDF boundaries far less often than that; more excuses would mean a systematic error
    hiding under the allowance."""
    return max(1, n_rows // 256)


def boundary_gap(oracle, row, params, hist, mask, u) -> dict | None:
    """Why a sampled token may differ from the reference's: the kind of decision boundary within
    BOUNDARY_EPS ("cdf": the uniform against the cumulative of the kept candidates; "top_p": the
    cumulative against top_p at the cut; "min_p": a probability ratio against min_p) and its
    distance, or None when no boundary is that close."""
    p = dict(zip(params.dtype.names, params[0]))
    if float(p["temperature"]) <= 0:
        return None
    st, ids, probs, n = oracle.candidates(row, params, hist, mask)
    if st != 0 or n == 0:
        return None
    cdf = np.cumsum(probs)
    d = np.abs(cdf - u)
    if d.min() < BOUNDARY_EPS:
        return {"kind": "cdf", "gap": float(d.min()), "at": int(d.argmin())}
    # top-p boundary: recompute the unrenormalised cumulative with top_p disabled
    q = params.copy()
    q["top_p"] = 1.0
    q["min_p"] = 0.0
    st2, ids2, probs2, n2 = oracle.candidates(row, q, hist, mask)
    tp = float(p["top_p"])
    if 0 < tp < 1 and st2 == 0:
        c2 = np.abs(np.cumsum(probs2) - tp)
        if c2.min() < BOUNDARY_EPS:
            return {"kind": "top_p", "gap": float(c2.min()), "at": int(c2.argmin())}
    mp = float(p["min_p"])
    if mp > 0 and st2 == 0 and n2 > 0:
        r = np.abs(probs2 / probs2[0] - mp)
        if r.min() < 1e-5:
            return {"kind": "min_p", "gap": float(r.min()), "at": int(r.argmin())}
    return None


def near_boundary(oracle, row, params, hist, mask, u, where: str = "") -> bool:
    """True when `u` lies within BOUNDARY_EPS of a CDF boundary of the reference distribution or
    when the top-p (min-p) decision is within BOUNDARY_EPS of flipping; every such excuse is
    recorded in EXCUSED with its kind and distance."""
    g = boundary_gap(oracle, row, params, hist, mask, u)
    if g is None:
        return False
    g["where"] = where
    EXCUSED.append(g)
    return True


def pytest_terminal_summary(terminalreporter):
    if not COMPARED["rows"] and not EXCUSED:
        return
    kinds: dict[str, int] = {}
    for e in EXCUSED:
        kinds[e["kind"]] = kinds.get(e["kind"], 0) + 1
    worst = max((e["gap"] for e in EXCUSED), default=0.0)
    terminalreporter.write_line(
        f"boundary excuses: {len(EXCUSED)} of {COMPARED['rows']} sampled rows compared with the oracle "
        f"({', '.join(f'{k} {v}' for k, v in sorted(kinds.items())) or 'none'}; largest gap {worst:.2e}, "
        f"allowance {BOUNDARY_EPS:g})")
