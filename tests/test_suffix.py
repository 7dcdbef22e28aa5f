"""CPU pinning of the suffix-drafter oracle (orc_suffix_draft) against the engine's own
SuffixDrafter (src/speculative/speculative.cpp:24-176, compiled into oracle/_ref): match lengths and
drafts, for propose and propose_anchored, must agree exactly."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import binding as B


def histories(rng, count):
    """Random histories over small and large vocabularies, with planted repeats, short ones and
    repetitive ones."""
    out = []
    for i in range(count):
        n = int(rng.choice([0, 1, 2, 3, 4, 5, 17, 40, 300, 2000, 20000]))
        vocab = int(rng.choice([2, 3, 5, 5, 64, 151_936]))
        h = rng.integers(0, vocab, size=n).astype(np.int32)
        if n > 60 and rng.random() < 0.8:  # plant a copy of the tail earlier in the history
            L = int(rng.integers(2, 24))
            at = int(rng.integers(0, n - 2 * L))
            h[at:at + L] = h[n - L:]
        out.append(h)
    return out


def test_port_matches_engine_drafter():
    ref = B.reference()
    if ref is None:
        pytest.skip("reference build absent")
    port = B.port()
    rng = np.random.default_rng(11)
    n_prop = 0
    for it, h in enumerate(histories(rng, 600)):
        min_match = int(rng.choice([0, 1, 2, 3, 4, 8, 17]))
        window = int(rng.choice([1, 8, 100, 16384]))
        k = int(rng.choice([0, 1, 4, 8, 50]))
        anchor = None
        if rng.random() < 0.4:
            anchor = int(h[rng.integers(0, h.size)]) if h.size and rng.random() < 0.8 else int(rng.integers(0, 64))
        a = port.suffix_draft(h, min_match, window, k, anchor)
        b = ref.suffix_draft(h, min_match, window, k, anchor)
        assert a[0] == b[0], (it, h.size, min_match, window, k, anchor, a[0], b[0])
        assert np.array_equal(a[1], b[1]), (it, a, b)
        n_prop += a[0] > 0
    assert n_prop > 40  # the cases exercise found proposals, not only misses


def test_engine_defaults_on_a_repeating_history():
    """SuffixDrafter(3, 16384): a history ending in a phrase seen before drafts its continuation."""
    port = B.port()
    h = np.array([5, 6, 7, 8, 9, 10, 11, 1, 2, 3, 5, 6, 7], np.int32)
    m, d = port.suffix_draft(h, 3, 16384, 4)
    assert m == 3 and d.tolist() == [8, 9, 10, 11]
    m, d = port.suffix_draft(h, 3, 16384, 4, anchor=8)  # pattern [.., 6, 7, 8]
    assert m >= 3 and d.tolist() == [9, 10, 11, 1]
