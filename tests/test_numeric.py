"""CPU pinning of the NaN / Inf policy oracle (orc_numeric_policy) against the engine.

The port (oracle/sixi_oracle.c) restates inspect_and_apply_numeric_policy
(src/core/numeric.cpp:628-699); the reference build (oracle/_ref) calls the engine's own function.
Both must reproduce the engine's unit test (tests/test_routing_and_numerics.cpp:415-460) and agree
with each other bit for bit, reports and rewritten rows, on random rows for both policies.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import binding as B

FAIL, CLAMP = 0, 1
NAN_OR_INF = 16


def impls():
    out = [B.port()]
    ref = B.reference()
    if ref is not None:
        out.append(ref)
    return out


@pytest.mark.parametrize("impl", impls(), ids=lambda o: o.kind)
def test_engine_unit_vectors(impl):
    """test_routing_and_numerics.cpp:415-460: cases 1 (fail) and 2 (clamp)."""
    d = np.array([1.0, 2.5, np.nan, -3.0, np.inf], np.float32)
    st, r = impl.numeric_policy(d, FAIL, 100.0)
    assert st == NAN_OR_INF and r["status"] == NAN_OR_INF
    assert not r["healthy"] and r["request_corrupted"] and r["state_invalidated"] and not r["emergency_clamped"]
    assert r["nan_count"] == 1 and r["inf_count"] == 1 and r["first_bad_index"] == 2
    assert np.isnan(d[2])  # never silently zeroed

    d = np.array([1.0, np.nan, np.inf, -np.inf, 500.0], np.float32)
    st, r = impl.numeric_policy(d, CLAMP, 100.0)
    assert st == 0 and r["emergency_clamped"] and r["nan_count"] == 1 and r["inf_count"] == 2
    assert np.isfinite(d).all() and (np.abs(d) <= 100.0).all()
    assert d.tolist() == [1.0, 0.0, 100.0, -100.0, 100.0]


def random_row(rng, n):
    x = rng.normal(0.0, 50.0, size=n).astype(np.float32)
    kind = rng.integers(0, 4)
    if kind >= 1:
        k = int(rng.integers(1, 6))
        idx = rng.choice(n, size=min(k, n), replace=False)
        x[idx] = rng.choice(np.array([np.nan, np.inf, -np.inf, -np.nan], np.float32), size=idx.size)
    if kind == 3:
        x[rng.integers(0, n)] = np.float32(3.0e38)
    return x


def test_port_matches_reference_bit_for_bit():
    ref = B.reference()
    if ref is None:
        pytest.skip("reference build absent")
    port = B.port()
    rng = np.random.default_rng(5)
    for it in range(400):
        n = int(rng.choice([0, 1, 5, 33, 1000, 4097]))
        x = random_row(rng, n) if n else np.zeros(0, np.float32)
        policy = int(rng.integers(0, 2))
        clamp = float(rng.choice(np.array([0.0, 100.0, -50.0, 3.5, np.inf, 1e-40], np.float32)))
        a, b = x.copy(), x.copy()
        sa, ra = port.numeric_policy(a, policy, clamp)
        sb, rb = ref.numeric_policy(b, policy, clamp)
        assert sa == sb, (it, sa, sb)
        assert ra.tobytes() == rb.tobytes(), (it, ra, rb)
        assert a.view(np.uint32).tolist() == b.view(np.uint32).tolist(), it
