"""GPU parity of the fused sampler kernels against the CPU oracle (calls through the C ABI).

Bars: greedy tokens, candidate id sets/order, masked sets and statuses bit-exact; sampled ids
exact except where the uniform is within 1e-6 of a reference CDF boundary; probabilities within
1e-5 relative (conftest.BOUNDARY_EPS / PROB_RTOL).
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import COMPARED, PROB_RTOL, has_gpu, max_excused, near_boundary

pytestmark = pytest.mark.gpu

if not has_gpu():  # collected on CPU boxes, skipped there
    pytest.skip("no CUDA device", allow_module_level=True)

import torch  # noqa: E402

import sixi_smp as S  # noqa: E402
from sixi_smp import workloads as W  # noqa: E402

DEV = torch.device("cuda:0")


def dev(a: np.ndarray | None):
    if a is None:
        return None
    if a.dtype.names is not None:  # params records
        return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8)).to(DEV)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(DEV)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(DEV).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


_samplers: dict[int, S.Sampler] = {}


def sampler(vocab: int) -> S.Sampler:
    if vocab not in _samplers:
        _samplers[vocab] = S.Sampler(0, 1024, vocab)
    return _samplers[vocab]


def run_sample(d: dict, uniforms: np.ndarray | None, step: int = 0):
    logits = d["logits"]
    vocab = d.get("vocab", logits.shape[1])
    smp = sampler(vocab)
    tok, st = smp.sample(dev(logits), dev(d["params"]), masks=dev(d.get("masks")), hist=dev(d.get("hist")),
                         hist_off=dev(d.get("hist_off")) if d.get("hist") is not None else None,
                         uniforms=dev(uniforms), step=step)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), st.cpu().numpy()


def check_against_oracle(port, d: dict, uniforms: np.ndarray, tok, st, step: int = 0):
    logits = d["logits"]
    vocab = d.get("vocab", logits.shape[1])
    if uniforms is None:
        uniforms = np.array([port.philox_uniform(int(p["seed"]), int(p["counter"]) + step, 0) for p in d["params"]])
    otok, ost = port.sample_batch(logits, d["params"], d.get("masks"), d.get("hist"), d.get("hist_off"),
                                  uniforms, step=step, vocab=vocab)
    assert np.array_equal(st, ost), f"status mismatch gpu={st} oracle={ost}"
    COMPARED["rows"] += int(len(tok))
    bad = np.nonzero(tok != otok)[0]
    excused = 0
    for r in bad:
        h = None
        if d.get("hist") is not None:
            h = d["hist"][d["hist_off"][r]:d["hist_off"][r + 1]]
        m = None
        if d.get("masks") is not None and (d["params"]["flags"][r] & S.ROW_MASKED):
            m = d["masks"][r]
        row = logits[r, :vocab]
        if near_boundary(port, row, d["params"][r:r + 1], h, m, uniforms[r], where=f"row {r}"):
            excused += 1
            continue
        raise AssertionError(f"row {r}: gpu token {tok[r]} oracle {otok[r]} params {d['params'][r]}")
    assert excused <= max_excused(len(tok)), f"{excused} boundary excuses over {len(tok)} rows"
    return excused


@pytest.mark.parametrize("seed", [11, 12, 13])
def test_config2_batched_sampler(port, seed):
    d = W.config2(rows=32, seed=seed)
    u = np.random.default_rng(seed).random(32)
    tok, st = run_sample(d, u)
    check_against_oracle(port, d, u, tok, st)


@pytest.mark.parametrize("seed", [21, 22])
def test_config3_grammar_masked(port, seed):
    d = W.config3(rows=32, seed=seed)
    u = np.random.default_rng(seed).random(32)
    tok, st = run_sample(d, u)
    check_against_oracle(port, d, u, tok, st)
    # every sampled token is allowed by its row's mask
    allowed = W.unpack_mask(d["masks"], d["logits"].shape[1])
    for r in range(32):
        assert st[r] == 0 and allowed[r, tok[r]]


def test_config1_single_row_philox(port):
    for greedy in (False, True):
        d = W.config1(greedy=greedy)
        for step in range(4):
            tok, st = run_sample(d, None, step=step)
            check_against_oracle(port, d, None, tok, st, step=step)


def rand_small_case(rng: np.random.Generator, vocab: int, rows: int, dtype: str):
    kind = rng.integers(0, 3)
    if kind == 0:
        logits = rng.normal(0.0, 2.5, size=(rows, vocab)).astype(np.float32)
    elif kind == 1:  # heavy ties
        logits = rng.integers(-3, 4, size=(rows, vocab)).astype(np.float32)
    else:
        logits = (rng.standard_cauchy(size=(rows, vocab)) * 0.5).astype(np.float32)
    if dtype == "bf16":
        bits = W.f32_to_bf16_bits(logits)
        logits_in = bits
    else:
        logits_in = logits
    t = rng.choice(np.array([0.0, 0.3, 0.7, 1.0, 1.5, 4.0], np.float32), size=rows)
    topk = rng.choice(np.array([0, 1, 2, 5, 20, 100, 256, 257, 300, 1000, vocab], np.int64), size=rows)
    topp = rng.choice(np.array([1.0, 0.95, 0.8, 0.5, 0.1], np.float32), size=rows)
    minp = np.where(rng.random(rows) < 0.2, rng.choice(np.array([0.01, 0.1, 0.5], np.float32), size=rows), 0.0)
    rep = rng.choice(np.array([1.0, 1.1, 1.3, 0.8], np.float32), size=rows)
    pres = np.where(rng.random(rows) < 0.3, 0.5, 0.0).astype(np.float32)
    freq = np.where(rng.random(rows) < 0.2, 0.25, 0.0).astype(np.float32)
    mode = np.where(rng.random(rows) < 0.8, S.ADAPTIVE, S.STRICT_REPLAY)
    params = S.make_params(rows, temperature=t, top_k=topk.astype(np.int32), top_p=topp, min_p=minp,
                           repetition_penalty=rep, presence_penalty=pres, frequency_penalty=freq, mode=mode)
    masks = None
    if rng.random() < 0.5:
        allowed = np.stack([W.run_mask(rng, vocab, float(rng.choice([0.05, 0.3, 0.9])), mean_run=4.0)
                            for _ in range(rows)])
        masks = W.pack_mask(allowed)
        params["flags"] = np.where(rng.random(rows) < 0.7, S.ROW_MASKED, 0)
    lens = rng.integers(0, 3 * vocab + 2, size=rows)
    off = np.zeros(rows + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    hist = rng.integers(-2, vocab + 2, size=int(off[-1]), dtype=np.int32)  # includes out-of-range ids
    return dict(logits=logits_in, params=params, masks=masks, hist=hist if off[-1] > 0 else None,
                hist_off=off if off[-1] > 0 else None, vocab=vocab)


@pytest.mark.parametrize("vocab", [1, 7, 31, 32, 33, 100, 513, 4097, 5000, 40000])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_small_vocab_random_params(port, vocab, dtype):
    rng = np.random.default_rng(vocab * 7 + (dtype == "bf16"))
    for it in range(3):
        d = rand_small_case(rng, vocab, 24, dtype)
        u = rng.random(24)
        tok, st = run_sample(d, u)
        check_against_oracle(port, d, u, tok, st)


def test_statuses_nan_inf_all_masked(port):
    vocab = 5000
    rng = np.random.default_rng(5)
    logits = rng.normal(0, 1, size=(6, vocab)).astype(np.float32)
    logits[0, 17] = np.nan
    logits[1, 4999] = np.inf
    logits[2, 0] = -np.inf
    allowed = np.ones((6, vocab), dtype=bool)
    allowed[3] = False                      # all masked
    allowed[4] = False
    allowed[4, 17] = True                   # single allowed token
    logits[5, 10] = np.nan
    allowed[5, 10] = False                  # NaN only on a masked token: fine
    params = S.make_params(6, temperature=0.8, top_k=0, top_p=0.9, flags=S.ROW_MASKED)
    d = dict(logits=logits, params=params, masks=W.pack_mask(allowed))
    u = rng.random(6)
    tok, st = run_sample(d, u)
    assert list(st) == [16, 16, 16, 1, 0, 0]
    assert tok[3] == -1 and tok[4] == 17
    check_against_oracle(port, d, u, tok, st)


def test_greedy_argmax_raw(port):
    vocab = 151_936
    rng = np.random.default_rng(3)
    x = rng.normal(0, 2.5, size=(8, vocab)).astype(np.float32)
    x[1, :] = 0.0                            # all tied -> 0
    x[2, 5] = x[2, 77] = x[2, 151_000] = 50.0  # tie -> 5
    x[3, 0] = np.nan                         # engine quirk: NaN at index 0 -> 0
    x[4, 100] = np.nan                       # other NaNs never win
    x[5, 151_935] = 1e30
    x[6, 3] = -0.0
    x[6, :] = np.minimum(x[6, :], -1.0)
    x[6, 3] = 0.0
    x[6, 2] = -0.0                           # -0 and +0 tie -> lower id
    smp = sampler(vocab)
    tok, st = smp.greedy_argmax(dev(x))
    tok = tok.cpu().numpy()
    st = st.cpu().numpy()
    for r in range(8):
        ost, otok = port.greedy_row(x[r])
        assert tok[r] == otok, (r, tok[r], otok)
        assert st[r] == ost
    assert tok[1] == 0 and tok[2] == 5 and tok[3] == 0 and tok[6] == 2


@pytest.mark.parametrize("seed", [31, 32])
def test_candidates_full_vocab(port, seed):
    d = W.config2(rows=16, seed=seed)
    d["params"]["temperature"] = np.where(d["params"]["temperature"] <= 0, 0.9, d["params"]["temperature"])
    smp = sampler(d["logits"].shape[1])
    ids, probs, cnt, st = smp.candidates(dev(d["logits"]), dev(d["params"]), max_out=256, hist=dev(d["hist"]),
                                         hist_off=dev(d["hist_off"]))
    ids, probs, cnt, st = (t.cpu().numpy() for t in (ids, probs, cnt, st))
    for r in range(16):
        h = d["hist"][d["hist_off"][r]:d["hist_off"][r + 1]]
        ost, oids, oprobs, on = port.candidates(d["logits"][r], d["params"][r:r + 1], h)
        assert st[r] == ost == 0
        assert cnt[r] == on, (r, cnt[r], on, d["params"][r])
        m = min(on, 256)
        assert np.array_equal(ids[r, :m], oids[:m]), r
        np.testing.assert_allclose(probs[r, :m], oprobs[:m], rtol=PROB_RTOL, atol=1e-300)


def test_philox_matches_host():
    vals = [S.philox_uniform(123, 7, s) for s in range(4)]
    from oracle import binding

    p = binding.port()
    assert vals == [p.philox_uniform(123, 7, s) for s in range(4)]


@pytest.mark.parametrize("vocab", [262_144, 600_000])
def test_wide_clusters_heavy_ties(port, vocab):
    """Clusters of 8 and 16 CTAs per row on integer-valued rows: the key-digit refine pass and the
    owner search of a crossing tie run over more CTAs."""
    rng = np.random.default_rng(vocab + 5)
    rows = 8
    logits = rng.integers(-3, 4, size=(rows, vocab)).astype(np.float32)
    W.boost_rows(rng, logits, n=4, by=3.0)
    params = S.make_params(rows, temperature=rng.choice(np.array([0.5, 1.0, 3.0], np.float32), size=rows),
                           top_k=np.array([0, 0, 300, 1000, 5000, 0, 257, 0], np.int32),
                           top_p=rng.choice(np.array([1.0, 0.9, 0.6], np.float32), size=rows))
    d = dict(logits=logits, params=params, masks=None, hist=None, hist_off=None, vocab=vocab)
    u = rng.random(rows)
    tok, st = run_sample(d, u)
    check_against_oracle(port, d, u, tok, st)


@pytest.mark.parametrize("vocab", [200_003, 262_144, 600_000])
def test_large_vocab_wide_clusters(port, vocab):
    """Vocabularies that need clusters of 8 (262,144) and 16 (600,000) CTAs per row."""
    rng = np.random.default_rng(vocab)
    rows = 6
    d = rand_small_case(rng, vocab, rows, "f32")
    lens = rng.integers(0, 3000, size=rows)
    off = np.zeros(rows + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    d["hist"] = rng.integers(-2, vocab + 2, size=int(off[-1]), dtype=np.int32)
    d["hist_off"] = off
    u = rng.random(rows)
    tok, st = run_sample(d, u)
    check_against_oracle(port, d, u, tok, st)
    smp = sampler(vocab)
    g, gs = smp.greedy_argmax(dev(d["logits"]))
    torch.cuda.synchronize()
    for r in range(rows):
        assert int(g[r]) == port.greedy_argmax(d["logits"][r]), r


@pytest.mark.parametrize("vocab", [7, 4097, 151_936])
def test_full_distribution(port, vocab):
    """sixi_smp_full_distribution against the restatement of compute_full_distribution."""
    rng = np.random.default_rng(vocab + 5)
    rows = 12
    x = rng.normal(0, 3, size=(rows, vocab)).astype(np.float32)
    temps = rng.choice(np.array([0.0, 0.25, 0.8, 1.0, 3.0], np.float32), size=rows)
    if vocab > 10:
        x[1, 5] = np.nan          # sampled row with a NaN: all zeros
        temps[1] = 1.0
        x[2, 0] = np.nan          # greedy row with a NaN at index 0: one-hot at 0
        temps[2] = 0.0
        x[3, rng.integers(0, vocab, size=4)] = -np.inf
        temps[3] = 0.7
        x[4, 9] = np.inf          # +inf: all zeros
        temps[4] = 0.5
    smp = sampler(vocab)
    for dt in ("f32", "bf16"):
        xin = x if dt == "f32" else W.f32_to_bf16_bits(x)
        got = smp.full_distribution(dev(xin), torch.from_numpy(temps).to(DEV)).cpu().numpy()
        for r in range(rows):
            want = port.full_distribution(xin[r], float(temps[r]))
            if temps[r] <= 0 or not np.any(want):
                assert np.array_equal(got[r], want), (dt, r)
            else:
                np.testing.assert_allclose(got[r], want, rtol=1e-6, atol=1e-30, err_msg=f"{dt} row {r}")


def mass_sweep_case(seed: int, dtype: str = "f32") -> dict:
    """32 full-vocabulary rows that mostly take the mass path (top_k = 0 or above the list limit):
    normal rows, integer-valued rows (heavy ties: bins far fuller than a gather segment) and
    Cauchy rows, each with 8 ids boosted by +6, a temperature / top-k / top-p / min-p mix,
    penalties, histories and, for 30 % of the rows, a run-structured mask."""
    vocab = W.QWEN_VOCAB
    rng = np.random.default_rng(seed)
    rows = 32
    kind = rng.integers(0, 3, size=rows)
    logits = np.empty((rows, vocab), np.float32)
    for r in range(rows):
        if kind[r] == 0:
            logits[r] = rng.normal(0.0, 2.5, size=vocab)
        elif kind[r] == 1:
            logits[r] = rng.integers(-4, 5, size=vocab)
        else:
            logits[r] = rng.standard_cauchy(size=vocab) * 0.7
    W.boost_rows(rng, logits, n=8, by=6.0)
    t = rng.choice(np.array([0.0, 0.35, 0.7, 1.0, 1.3, 3.0], np.float32), size=rows)
    topk = rng.choice(np.array([0, 0, 0, 300, 1000, 40], np.int32), size=rows)
    topp = rng.choice(np.array([1.0, 0.99, 0.9, 0.75, 0.3], np.float32), size=rows)
    minp = np.where(rng.random(rows) < 0.25, rng.choice(np.array([0.001, 0.05], np.float32), size=rows), 0.0)
    params = S.make_params(rows, temperature=t, top_k=topk, top_p=topp, min_p=minp,
                           repetition_penalty=rng.choice(np.array([1.0, 1.2], np.float32), size=rows),
                           presence_penalty=np.where(rng.random(rows) < 0.3, 0.4, 0.0).astype(np.float32))
    allowed = np.stack([W.run_mask(rng, vocab, float(rng.choice([0.02, 0.5])), mean_run=64.0)
                        for _ in range(rows)])
    masks = W.pack_mask(allowed)
    params["flags"] = np.where(rng.random(rows) < 0.3, S.ROW_MASKED, 0)
    lens = rng.integers(0, 2048, size=rows)
    off = np.zeros(rows + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32)
    if dtype == "bf16":
        logits = W.f32_to_bf16_bits(logits)
    d = dict(logits=logits, params=params, masks=masks, hist=hist, hist_off=off, vocab=vocab)
    d["uniforms"] = rng.random(rows)
    return d


@pytest.mark.parametrize("seed", [41, 42, 43])
def test_full_vocab_mass_path_sweep(port, seed):
    """The exact selections over one to hundreds of entries, the bin-boundary search, the gather
    pass and the key-digit refine pass, on full-vocabulary rows."""
    d = mass_sweep_case(seed)
    tok, st = run_sample(d, d["uniforms"])
    check_against_oracle(port, d, d["uniforms"], tok, st)


@pytest.mark.parametrize("seed", [44, 45])
def test_full_vocab_mass_path_sweep_bf16(port, seed):
    d = mass_sweep_case(seed, "bf16")
    tok, st = run_sample(d, d["uniforms"])
    check_against_oracle(port, d, d["uniforms"], tok, st)


@pytest.mark.parametrize("seed", [46, 47])
def test_candidates_full_vocab_mass_path(port, seed):
    """Candidate lists (ids, order, probabilities and the kept count) of the sweep's rows, the
    greedy rows given a temperature."""
    d = mass_sweep_case(seed)
    d["params"]["temperature"] = np.where(d["params"]["temperature"] <= 0, 0.8, d["params"]["temperature"])
    rows = d["logits"].shape[0]
    smp = sampler(d["vocab"])
    ids, probs, cnt, st = smp.candidates(dev(d["logits"]), dev(d["params"]), max_out=256, masks=dev(d["masks"]),
                                         hist=dev(d["hist"]), hist_off=dev(d["hist_off"]))
    ids, probs, cnt, st = (t.cpu().numpy() for t in (ids, probs, cnt, st))
    masks = d["masks"]
    for r in range(rows):
        h = d["hist"][d["hist_off"][r]:d["hist_off"][r + 1]]
        m_r = masks[r] if d["params"]["flags"][r] & S.ROW_MASKED else None
        ost, oids, oprobs, on = port.candidates(d["logits"][r], d["params"][r:r + 1], h, mask=m_r)
        assert st[r] == ost, (r, st[r], ost)
        if ost != 0:
            continue
        assert cnt[r] == on, (r, cnt[r], on, d["params"][r])
        m = min(on, 256)
        assert np.array_equal(ids[r, :m], oids[:m]), r
        np.testing.assert_allclose(probs[r, :m], oprobs[:m], rtol=PROB_RTOL, atol=1e-300)

@pytest.mark.parametrize("seed", [51, 52])
def test_kbound_inside_overfull_tie_bin(port, seed):
    """Integer-valued logits put thousands of equal keys in one bin, so the k-th entry of a
    top_k above the list limit is found by the key-digit refine pass in counting mode. The kept
    mass that follows must weigh each tie by its own weight, not by one, or every later target
    (top-p, min-p, the draw) moves."""
    vocab = W.QWEN_VOCAB
    rng = np.random.default_rng(seed)
    rows = 24
    logits = rng.integers(-3, 4, size=(rows, vocab)).astype(np.float32)
    W.boost_rows(rng, logits, n=4, by=3.0)
    t = rng.choice(np.array([0.5, 1.3, 3.0], np.float32), size=rows)
    topk = rng.choice(np.array([257, 300, 1000, 5000], np.int32), size=rows)
    topp = rng.choice(np.array([1.0, 0.9, 0.6], np.float32), size=rows)
    params = S.make_params(rows, temperature=t, top_k=topk, top_p=topp)
    d = dict(logits=logits, params=params, masks=None, hist=None, hist_off=None)
    u = rng.random(rows)
    tok, st = run_sample(d, u)
    check_against_oracle(port, d, u, tok, st)


@pytest.mark.parametrize("seed", [71, 72])
def test_full_vocab_extreme_parameters(port, seed):
    """Temperatures from 1e-3 (every weight but the largest rounds to zero) to 1,000 (every weight
    close to the largest), top_p and min_p at their limits, top_k at 1, just above the list limit
    and at the vocabulary size, on normal, integer-valued and Cauchy rows."""
    vocab = W.QWEN_VOCAB
    rng = np.random.default_rng(seed)
    rows = 32
    logits = np.empty((rows, vocab), np.float32)
    for r in range(rows):
        if r % 3 == 0:
            logits[r] = rng.normal(0.0, 2.5, size=vocab)
        elif r % 3 == 1:
            logits[r] = rng.integers(-2, 3, size=vocab)
        else:
            logits[r] = rng.standard_cauchy(size=vocab) * 3.0
    t = rng.choice(np.array([1e-3, 0.05, 20.0, 1000.0], np.float32), size=rows)
    topk = rng.choice(np.array([0, 0, 1, 257, vocab - 1, vocab], np.int32), size=rows)
    topp = rng.choice(np.array([1.0, 0.999999, 1e-6, 0.5], np.float32), size=rows)
    minp = rng.choice(np.array([0.0, 0.0, 1e-9, 0.999], np.float32), size=rows)
    params = S.make_params(rows, temperature=t, top_k=topk, top_p=topp, min_p=minp)
    d = dict(logits=logits, params=params, masks=None, hist=None, hist_off=None)
    u = rng.random(rows)
    u[:4] = [0.0, 1.0 - 2.0 ** -53, 0.5, 1e-12]  # the ends of the unit interval
    tok, st = run_sample(d, u)
    check_against_oracle(port, d, u, tok, st)


@pytest.mark.parametrize("seed", [81, 82, 83])
def test_topp_cut_position_on_mass_path(port, seed):
    """The top-p cut of rows on the mass path (top_k = 0, config-2 temperatures and top_p) is decided
    on fixed-point weights built from ex2.approx: the kept count must equal the engine's on every
    row whose cumulative at the cut is further than 1e-6 from top_p, and rows closer than that stay
    within the excuse bound. The smallest distance seen is printed, so the margin is on record."""
    rows = 64
    d = W.config2(rows=rows, seed=seed)
    d["params"]["top_k"] = 0
    d["params"]["temperature"] = np.where(d["params"]["temperature"] <= 0, 0.9, d["params"]["temperature"])
    smp = sampler(W.QWEN_VOCAB)
    _, _, cnt, st = smp.candidates(dev(d["logits"]), dev(d["params"]), max_out=1, hist=dev(d["hist"]),
                                   hist_off=dev(d["hist_off"]))
    cnt, st = cnt.cpu().numpy(), st.cpu().numpy()
    excused, gaps = 0, []
    for r in range(rows):
        h = d["hist"][d["hist_off"][r]:d["hist_off"][r + 1]]
        q = d["params"][r:r + 1].copy()
        tp = float(q["top_p"][0])
        q["top_p"] = 1.0
        ost, _, oprobs, on = port.candidates(d["logits"][r], q, h)
        assert st[r] == 0 and ost == 0
        cum = np.cumsum(oprobs)
        keep = min(int(np.searchsorted(cum, tp) + 1), int(on))  # first cum >= top_p, crossing kept
        gap = float(np.abs(cum[max(0, keep - 2):keep + 1] - tp).min())
        gaps.append(gap)
        if cnt[r] != keep:
            assert gap < 1e-6, (r, cnt[r], keep, gap)
            excused += 1
    print(f"top-p cuts: {rows} rows, {excused} within 1e-6 of top_p and moved, smallest gap {min(gaps):.2e}")
    assert excused <= max_excused(rows)


def test_sample_host_async_pipelined_batches(port):
    """sixi_smp_sample_host_async: five config-2 batches queued back to back (two staging slots, so
    batch i+1's copy overlaps batch i's kernel), one synchronisation at the end; every batch's
    tokens and statuses equal the blocking host call's and the oracle's."""
    rows = 16
    smp = S.Sampler(0, 64, W.QWEN_VOCAB)
    stream = torch.cuda.Stream(device=DEV)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()  # noqa: E731
    ds = [W.config2(rows=rows, seed=900 + i) for i in range(5)]
    us = [np.random.default_rng(900 + i).random(rows) for i in range(5)]
    ins = [(pin(d["logits"]), pin(d["params"].view(np.uint8)).view(S.PARAMS_DTYPE), pin(d["hist"]),
            pin(d["hist_off"]), pin(u)) for d, u in zip(ds, us)]
    outs = [(pin(np.full(rows, -7, np.int32)), pin(np.full(rows, -7, np.int32))) for _ in ds]
    for (lg, prm, h, ho, u), (tok, st) in zip(ins, outs):
        smp.sample_host(lg, prm, hist=h, hist_off=ho, uniforms=u, out_tokens=tok, out_status=st, stream=stream,
                        wait=False)
    stream.synchronize()
    for (lg, prm, h, ho, u), (tok, st), d in zip(ins, outs, ds):
        t2, s2 = smp.sample_host(lg, prm, hist=h, hist_off=ho, uniforms=u, stream=stream)
        assert np.array_equal(tok, t2) and np.array_equal(st, s2)
        check_against_oracle(port, d, u, tok, st)
    smp.close()
