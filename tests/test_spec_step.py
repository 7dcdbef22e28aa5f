"""The verifier restatement pinned to the engine's own SpeculativeDecoder::step.

The reference build (oracle/_ref) runs the engine's step() through a replay IBackend (pre-supplied
target rows) and a fixed-draft INeuralDrafter, with the engine's DeterministicRng:
  slow path  no rollback ring, dense draft probabilities (src/speculative/speculative.cpp:739-976)
  fast path  O(1) rollback, one-hot drafts after an anchor drawn from the previous logits (:471-737)
The port's verifier (orc_verify, the checker of every GPU verify test) is given the uniforms the
engine's RNG yields, in order, and must commit the same tokens, accept the same number of drafts,
reject at the same position and consume exactly the uniforms that leave the engine's RNG in the
state step() leaves it. Cases: config-4 rows (bf16 target ~ N(0, 3^2), q = softmax of target plus
N(0, 1) noise), sampled and greedy, and a forced rejection at every draft position.
"""

from __future__ import annotations

import numpy as np
import pytest

from sixi_smp import workloads as W

K = 8


@pytest.fixture(scope="module")
def ref(reference):
    if not hasattr(reference.lib, "orc_ref_spec_step"):
        pytest.skip("reference build without the decoder entry points")
    return reference


def _case(vocab, seed, greedy=False):
    d = W.config4(streams=2, k=K, vocab=vocab, seed=seed, stochastic=not greedy, masked=False)
    rows = W.bf16_bits_to_f32(d["target_bits"]).reshape(2, K + 1, vocab)
    q = d["q"].reshape(2, K, vocab)
    return d, rows, q


def _port_verify(port, rows, drafts, prm, q, hist, uniforms):
    S = 1
    hoff = np.array([0, hist.size], dtype=np.int64)
    u = np.zeros((S, K + 1))
    u[0, :len(uniforms)] = uniforms[:K + 1]
    out = port.verify(rows.reshape(K + 1, -1), drafts.reshape(1, K), prm, q=q, hist=hist, hist_off=hoff, uniforms=u)
    n = int(out["n_tokens"][0])
    return dict(tokens=out["tokens"][0, :n].copy(), accepted=int(out["accepted"][0]),
                first_reject=int(out["first_reject"][0]), used=int(out["uniforms_used"][0]),
                status=int(out["status"][0]))


def _check_slow(port, ref, rows, drafts, prm, q, hist, seed):
    st0 = ref.rng_seed(seed)
    uni = ref.rng_uniforms(st0.copy(), K + 1)
    eng = ref.spec_step(rows, drafts, prm, hist=hist, draft_probs=q, rng_state=st0.copy())
    mine = _port_verify(port, rows, drafts, prm, q, hist, uni)
    assert eng["status"] == 0 and mine["status"] == 0
    assert np.array_equal(eng["tokens"], mine["tokens"]), (eng, mine)
    assert eng["accepted"] == mine["accepted"] and eng["first_reject"] == mine["first_reject"], (eng, mine)
    after = st0.copy()
    ref.rng_uniforms(after, mine["used"])
    assert np.array_equal(after, eng["rng"]), "RNG state after step differs from the uniforms the verifier used"
    return eng


@pytest.mark.parametrize("vocab,seed", [(4097, 1), (4097, 2), (33, 3), (151_936, 4)])
def test_slow_path_dense_q_matches_engine_step(port, ref, vocab, seed):
    d, rows, q = _case(vocab, seed)
    for s in range(2):
        h = d["hist"][d["hist_off"][s]:d["hist_off"][s + 1]]
        _check_slow(port, ref, rows[s], d["drafts"][s], d["params"][s:s + 1], q[s], h, 1000 * seed + s)


@pytest.mark.parametrize("vocab,seed", [(4097, 5), (151_936, 6)])
def test_slow_path_greedy_matches_engine_step(port, ref, vocab, seed):
    d, rows, q = _case(vocab, seed, greedy=True)
    for s in range(2):
        h = d["hist"][d["hist_off"][s]:d["hist_off"][s + 1]]
        # drafts: the raw argmax of the first half of the rows, so that some are accepted
        dr = d["drafts"][s].copy()
        for i in range(K // 2):
            dr[i] = int(np.argmax(rows[s, i]))
        eng = _check_slow(port, ref, rows[s], dr, d["params"][s:s + 1], q[s], h, 77 + s)
        assert eng["accepted"] >= K // 2


@pytest.mark.parametrize("greedy", [False, True])
def test_forced_rejection_at_every_position(port, ref, greedy):
    vocab = 4097
    d, rows, q = _case(vocab, 11, greedy=greedy)
    prm = d["params"][:1].copy()
    h = d["hist"][d["hist_off"][0]:d["hist_off"][1]]
    for j in range(K):
        dr = d["drafts"][0].copy()
        qq = q[0].copy()
        recent = list(h)
        for i in range(K):
            row = rows[0, i]
            if greedy:
                top = int(np.argmax(row))
                dr[i] = top if i < j else (top + 1) % vocab
                continue
            st, ids, probs, n = port.candidates(row, prm, hist=np.array(recent, dtype=np.int32))
            assert st == 0
            if i < j:
                dr[i] = ids[0]            # a kept candidate
                qq[i, dr[i]] = 1e-9       # q_d << p_d: accepted whatever the uniform
                recent.append(int(dr[i]))
            elif i == j:
                outside = np.setdiff1d(np.arange(vocab), ids)
                dr[i] = int(outside[0])   # p_d = 0: rejected whatever the uniform
        eng = _check_slow(port, ref, rows[0], dr, prm, qq, h, 500 + j)
        assert eng["first_reject"] == j and eng["accepted"] == j, (j, eng)


@pytest.mark.parametrize("greedy", [False, True])
@pytest.mark.parametrize("vocab,seed", [(4097, 21), (151_936, 22)])
def test_fast_path_one_hot_matches_engine_step(port, ref, vocab, seed, greedy):
    """Fast path: the engine draws the anchor from the previous logits, verifies the one-hot drafts
    against the k + 1 rows after it and carries the replacement / bonus to the next step. The port
    draws the anchor with sample() (greedy: the raw argmax), then verifies with q = NULL and the
    anchor appended to the penalty history."""
    d, rows, q = _case(vocab, seed, greedy=greedy)
    rng = np.random.default_rng(seed)
    for s in range(2):
        h = d["hist"][d["hist_off"][s]:d["hist_off"][s + 1]]
        prm = d["params"][s:s + 1]
        anchor_row = (rng.normal(0.0, 3.0, size=vocab)).astype(np.float32)
        dr = d["drafts"][s].copy()
        for i in range(s * 3):  # stream 1: the first drafts are the rows' best, so some are accepted
            dr[i] = int(np.argmax(rows[s, i]))
        st0 = ref.rng_seed(seed * 10 + s)
        eng = ref.spec_step(rows[s], dr, prm, hist=h, rng_state=st0.copy(), fast=True, anchor_row=anchor_row)
        assert eng["status"] == 0
        mine_rng = st0.copy()
        if greedy:
            anchor = int(np.argmax(anchor_row))
        else:
            u0 = ref.rng_uniforms(mine_rng, 1)[0]
            sst, anchor = port.sample(anchor_row, prm, hist=h, u=u0)
            assert sst == 0
        uni = ref.rng_uniforms(mine_rng.copy(), K + 1)
        hist2 = np.concatenate([h, np.array([anchor], dtype=np.int32)])
        mine = _port_verify(port, rows[s], dr, prm, None, hist2, uni)
        assert mine["status"] == 0
        assert np.array_equal(eng["tokens"], np.concatenate([[anchor], mine["tokens"]])), (eng, anchor, mine)
        assert eng["accepted"] == mine["accepted"] and eng["first_reject"] == mine["first_reject"]
        ref.rng_uniforms(mine_rng, mine["used"])
        assert np.array_equal(mine_rng, eng["rng"])
