"""CPU tests of the oracle (the parity checker): Philox known answers, the C restatement against the
golden vectors the engine's own code produced, against the engine build itself on random cases,
and the semantic checks of the engine's sampler tests."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import REPO

import sixi_smp as S
from sixi_smp import workloads as W

GOLDEN = REPO / "tests" / "golden" / "golden.npz"


def test_philox_known_answers(port):
    """Random123 known-answer vectors of Philox4x32-10."""
    cases = [
        ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
        ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
        ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
         [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
    ]
    fn = port.lib.orc_philox4x32_10
    fn.restype = None
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    for ctr, key, want in cases:
        c = (ctypes.c_uint32 * 4)(*ctr)
        k = (ctypes.c_uint32 * 2)(*key)
        o = (ctypes.c_uint32 * 4)()
        fn(c, k, o)
        assert list(o) == want


def test_port_matches_golden(port):
    import golden.make_golden as G

    g = np.load(GOLDEN)
    for i, c in enumerate(G.cases()):
        st, ids, probs, n = port.candidates(c["logits"], c["params"], c["hist"], c["mask"])
        st2, tok = port.sample(c["logits"], c["params"], c["hist"], c["mask"], c["u"])
        assert [st, st2] == list(g[f"c{i}_status"]), i
        assert n == int(g[f"c{i}_n"][0]), i
        k = len(g[f"c{i}_ids"])
        assert np.array_equal(ids[:k], g[f"c{i}_ids"]), i
        np.testing.assert_allclose(probs[:k], g[f"c{i}_probs"], rtol=1e-12, atol=0)
        assert tok == int(g[f"c{i}_token"][0]), i
    for i, d in enumerate(G.verify_cases()):
        o = port.verify(d["target_bits"], d["drafts"], d["params"], q=d["q"] if d["dense"] else None,
                        masks=d["masks"], hist=d["hist"], hist_off=d["hist_off"], uniforms=d["uniforms"])
        for k2, v in o.items():
            assert np.array_equal(v, g[f"v{i}_{k2}"]), (i, k2, v, g[f"v{i}_{k2}"])
    assert port.greedy_argmax(np.array([-1.0, 5.5, 3.2, 5.5, 5.5, 0.0], np.float32)) == int(g["tie_argmax"][0]) == 1


def _random_row(rng, vocab):
    logits = rng.normal(0.0, float(rng.choice([0.5, 2.5, 6.0])), size=vocab).astype(np.float32)
    if rng.random() < 0.3:
        logits = np.round(logits * 2).astype(np.float32)
    p = S.make_params(1, temperature=float(rng.choice([0.0, 0.25, 0.7, 1.0, 2.0])),
                      top_k=int(rng.choice([0, 1, 3, 20, 100, 5000, vocab])),
                      top_p=float(rng.choice([1.0, 0.9, 0.5, 0.05])),
                      repetition_penalty=float(rng.choice([1.0, 1.2, 0.9])),
                      presence_penalty=float(rng.choice([0.0, 0.7, -0.3])),
                      mode=int(rng.choice([S.STRICT_REPLAY, S.ADAPTIVE])))
    hist = rng.integers(-3, vocab + 3, size=int(rng.integers(0, 200)), dtype=np.int32)
    mask = None
    if rng.random() < 0.4:
        mask = W.pack_mask(W.run_mask(rng, vocab, float(rng.choice([0.001, 0.1, 0.7])), mean_run=6.0)[None])[0]
        p["flags"] = S.ROW_MASKED
    return logits, p, hist, mask


@pytest.mark.parametrize("vocab", [1, 2, 31, 64, 1000, 20000])
def test_port_matches_reference_random(port, reference, vocab):
    rng = np.random.default_rng(vocab)
    for _ in range(40):
        logits, p, hist, mask = _random_row(rng, vocab)
        a = port.candidates(logits, p, hist, mask)
        b = reference.candidates(logits, p, hist, mask)
        assert a[0] == b[0] and a[3] == b[3]
        assert np.array_equal(a[1], b[1])
        np.testing.assert_array_equal(a[2], b[2])
        u = float(rng.random())
        assert port.sample(logits, p, hist, mask, u) == reference.sample(logits, p, hist, mask, u)


def test_port_matches_reference_verify(port, reference):
    for seed in range(5):
        for dense in (True, False):
            for stochastic in (True, False):
                d = W.config4(streams=5, k=3, vocab=700, seed=100 + seed, stochastic=stochastic, masked=seed % 2 == 0)
                kw = dict(q=d["q"] if dense else None, masks=d["masks"], hist=d["hist"], hist_off=d["hist_off"],
                          uniforms=d["uniforms"])
                a = port.verify(d["target_bits"], d["drafts"], d["params"], **kw)
                b = reference.verify(d["target_bits"], d["drafts"], d["params"], **kw)
                for k in a:
                    assert np.array_equal(a[k], b[k]), (seed, dense, stochastic, k)


def test_engine_sampler_unit_semantics(port):
    """The checks of the engine's test_sampler_candidates_topk_topp, on the restatement."""
    import golden.make_golden as G

    x = G.engine_test_logits()
    order = sorted(range(len(x)), key=lambda i: (-x[i], i))
    p = S.make_params(1, temperature=1.0, top_k=20, top_p=1.0, mode=S.STRICT_REPLAY)
    st, ids, probs, n = port.candidates(x, p)
    assert st == 0 and n == 20
    assert list(ids) == order[:20]
    assert np.all(np.diff(probs) <= 0) and abs(probs.sum() - 1.0) < 1e-9
    assert ids[0] == port.greedy_argmax(x)
    p["top_p"] = 0.5
    st, ids2, probs2, n2 = port.candidates(x, p)
    assert 0 < n2 < 20 and ids2[0] == order[0] and abs(probs2.sum() - 1.0) < 1e-9
    st, t1 = port.sample(x, p, u=0.37)
    assert t1 in set(ids2.tolist())
    p["temperature"] = 0.0
    st, tg = port.sample(x, p, u=0.99)
    assert tg == order[0]


def test_verify_forced_rejection_positions(port):
    """Greedy verification rejects exactly at the first wrong draft and commits the target argmax;
    full acceptance appends the bonus argmax (speculative.cpp:801-822)."""
    rng = np.random.default_rng(3)
    v, k = 256, 4
    tgt = rng.normal(0, 1, size=(1, k + 1, v)).astype(np.float32)
    am = tgt[0].argmax(axis=1).astype(np.int32)
    params = S.make_params(1, temperature=0.0)
    for pos in range(k + 1):
        drafts = am[:k].copy()[None]
        if pos < k:
            drafts[0, pos] = (am[pos] + 17) % v
        o = port.verify(tgt.reshape(k + 1, v), drafts, params, q=np.full((k, v), 1.0 / v, np.float32))
        assert o["accepted"][0] == pos
        assert o["first_reject"][0] == (pos if pos < k else -1)
        assert list(o["tokens"][0, :pos + 1]) == list(am[:pos + 1])
        assert o["uniforms_used"][0] == 0


def test_masked_tokens_never_sampled(port):
    rng = np.random.default_rng(9)
    d = W.config3(rows=6, vocab=3000, seed=4)
    u = rng.random(6)
    tok, st = port.sample_batch(d["logits"], d["params"], d["masks"], d["hist"], d["hist_off"], u)
    allowed = W.unpack_mask(d["masks"], 3000)
    assert all(st == 0) and all(allowed[r, tok[r]] for r in range(6))


def test_full_distribution_port_matches_reference(port, reference):
    """compute_full_distribution: the restatement against the engine's own function, including
    greedy one-hots, NaN / +inf rows (all zeros) and -inf entries."""
    rng = np.random.default_rng(17)
    for vocab in (1, 7, 1000, 40000):
        for t in (0.0, 0.3, 1.0, 2.5):
            for case in range(3):
                x = rng.normal(0, 3, size=vocab).astype(np.float32)
                if vocab > 10 and case == 1:
                    x[rng.integers(0, vocab)] = np.nan
                if vocab > 10 and case == 2:
                    x[rng.integers(0, vocab, size=5)] = -np.inf
                    x[0] = np.inf if t == 2.5 else x[0]
                a = port.full_distribution(x, t)
                b = reference.full_distribution(x, t)
                assert np.array_equal(a, b), (vocab, t, case)
    bits = W.f32_to_bf16_bits(rng.normal(0, 2, size=5000).astype(np.float32))
    assert np.array_equal(port.full_distribution(bits, 0.7), reference.full_distribution(bits, 0.7))
