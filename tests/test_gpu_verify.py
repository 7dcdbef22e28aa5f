"""GPU parity of the speculative verifier (sixi_smp_verify) against the CPU oracle.

Accept/reject decisions, committed tokens, first-reject positions and the number of uniforms
consumed are compared bit-exactly (speculative.cpp:801-916 for dense draft probabilities,
589-692 for one-hot drafts). The seeded inputs below place no decision within 1e-6 of a
boundary, so no mismatch is excused.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu

if not has_gpu():
    pytest.skip("no CUDA device", allow_module_level=True)

import torch  # noqa: E402

import sixi_smp as S  # noqa: E402
from sixi_smp import workloads as W  # noqa: E402
from test_gpu_parity import dev, sampler  # noqa: E402

KEYS = ("accepted", "tokens", "n_tokens", "first_reject", "uniforms_used", "status")


def run_verify(d: dict, dense: bool, uniforms="given", n_drafts=None, step: int = 0, bf16: bool = True):
    vocab = d["target_bits"].shape[1]
    target = d["target_bits"] if bf16 else W.bf16_bits_to_f32(d["target_bits"])
    u = d["uniforms"] if uniforms == "given" else None
    smp = sampler(vocab)
    o = smp.verify(dev(target), dev(d["drafts"]), dev(d["params"]), draft_probs=dev(d["q"]) if dense else None,
                   n_drafts=dev(n_drafts), masks=dev(d["masks"]), hist=dev(d["hist"]), hist_off=dev(d["hist_off"]),
                   uniforms=dev(u), step=step)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in o.items()}, target, u


def check(port, d: dict, dense: bool, uniforms="given", n_drafts=None, step: int = 0, bf16: bool = True):
    g, target, u = run_verify(d, dense, uniforms, n_drafts, step, bf16)
    o = port.verify(target, d["drafts"], d["params"], q=d["q"] if dense else None, n_drafts=n_drafts,
                    masks=d["masks"], hist=d["hist"], hist_off=d["hist_off"], uniforms=u, step=step)
    for k in KEYS:
        assert np.array_equal(g[k], o[k]), f"{k}: gpu={g[k]} oracle={o[k]}"
    return g


def test_verify_golden_vectors():
    """The engine-generated verify goldens, through the GPU."""
    import golden.make_golden as G

    g = np.load(G.OUT)
    for i, d in enumerate(G.verify_cases()):
        o, _, _ = run_verify(d, d["dense"])
        for k in KEYS:
            assert np.array_equal(o[k], g[f"v{i}_{k}"]), (i, k, o[k], g[f"v{i}_{k}"])


@pytest.mark.parametrize("dense", [True, False])
@pytest.mark.parametrize("stochastic", [True, False])
def test_verify_config4_full_vocab(port, dense, stochastic):
    """Config 4: 32 streams x 8 drafts, V=151,936 bf16 targets, parameter mix, grammar masks."""
    d = W.config4(streams=32, k=8, seed=41 + dense + 2 * stochastic, stochastic=stochastic, masked=True)
    g = check(port, d, dense)
    if stochastic:
        assert g["accepted"].min() >= 0 and g["accepted"].max() <= 8


@pytest.mark.parametrize("vocab", [1, 33, 700, 4097])
@pytest.mark.parametrize("dense", [True, False])
def test_verify_small_vocab(port, vocab, dense):
    for seed in range(3):
        d = W.config4(streams=5, k=3, vocab=vocab, seed=200 + seed, stochastic=seed != 1, masked=seed % 2 == 0)
        check(port, d, dense, bf16=seed != 2)


def test_verify_ragged_drafts_and_philox(port):
    """n_drafts below k for some streams, and uniforms drawn by the library (Philox slots 0..k)."""
    d = W.config4(streams=12, k=6, vocab=3000, seed=77, stochastic=True, masked=True)
    nd = np.array([6, 0, 1, 2, 3, 4, 5, 6, 0, 6, 3, 1], dtype=np.int32)
    check(port, d, True, n_drafts=nd)
    check(port, d, False, n_drafts=nd)
    check(port, d, True, uniforms=None, step=5)
    check(port, d, False, uniforms=None, step=9, n_drafts=nd)


def test_verify_greedy_forced_rejections(port):
    """Greedy match rejects exactly at the first wrong draft (engine test: forced rejection)."""
    rng = np.random.default_rng(3)
    v, k = 4096, 4
    tgt = rng.normal(0, 1, size=(k + 1, k + 1, v)).astype(np.float32)
    drafts = np.empty((k + 1, k), np.int32)
    for s in range(k + 1):
        am = tgt[s].argmax(axis=1)
        drafts[s] = am[:k]
        if s < k:
            drafts[s, s] = (am[s] + 17) % v
    params = S.make_params(k + 1, temperature=0.0)
    smp = sampler(v)
    o = smp.verify(dev(tgt.reshape(-1, v)), dev(drafts), dev(params))
    torch.cuda.synchronize()
    acc = o["accepted"].cpu().numpy()
    assert list(acc) == list(range(k + 1))
    ref = port.verify(tgt.reshape(-1, v), drafts, params)
    for key in KEYS:
        assert np.array_equal(o[key].cpu().numpy(), ref[key]), key


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_verify_draft_logits_equals_stored_q(port, dtype):
    """q evaluated from draft logits inside the verifier == q stored by full_distribution, then
    verified; both == the oracle (compute_full_distribution, then dense-q verification)."""
    d = W.config4(streams=8, k=4, vocab=151_936, seed=71, stochastic=True, masked=True)
    S_, k = d["streams"], d["k"]
    lg = d["draft_logits"].copy()
    temps = np.where(np.arange(S_ * k) % 5 == 0, 0.0, 0.6 + 0.1 * (np.arange(S_ * k) % 7)).astype(np.float32)
    lg[3, 1000] = np.nan  # a row whose distribution is all zero
    lg[6, :] = -np.inf  # no finite maximum: all zero as well
    if dtype == "bf16":
        lg_bits = W.f32_to_bf16_bits(lg)
        lg = W.bf16_bits_to_f32(lg_bits)
        d_lg = torch.from_numpy(lg_bits.view(np.int16)).to("cuda").view(torch.bfloat16)
    else:
        d_lg = dev(lg)
    # drafts from the evaluated q (one-hot rows draft their argmax, zero rows keep a random draft)
    smp = sampler(151_936)
    q = smp.full_distribution(d_lg, dev(temps))
    qh = q.cpu().numpy()
    drafts = d["drafts"].copy()
    for r in range(S_ * k):
        if temps[r] <= 0:
            drafts[r // k, r % k] = int(np.argmax(qh[r]))
    args = dict(n_drafts=None, masks=dev(d["masks"]), hist=dev(d["hist"]), hist_off=dev(d["hist_off"]),
                uniforms=dev(d["uniforms"]))
    tgt = dev(d["target_bits"])
    fused = smp.verify_draft_logits(tgt, d_lg, dev(temps), dev(drafts), dev(d["params"]), **args)
    stored = smp.verify(tgt, dev(drafts), dev(d["params"]), draft_probs=q, **args)
    torch.cuda.synchronize()
    fused = {kk: v.cpu().numpy() for kk, v in fused.items()}
    stored = {kk: v.cpu().numpy() for kk, v in stored.items()}
    for kk in KEYS:
        assert np.array_equal(fused[kk], stored[kk]), kk
    qo = np.stack([port.full_distribution(lg[r], float(temps[r])) for r in range(S_ * k)])
    o = port.verify(W.bf16_bits_to_f32(d["target_bits"]), drafts, d["params"], q=qo, masks=d["masks"],
                    hist=d["hist"], hist_off=d["hist_off"], uniforms=d["uniforms"])
    for kk in KEYS:
        assert np.array_equal(fused[kk], o[kk]), f"{kk}: gpu={fused[kk]} oracle={o[kk]}"


@pytest.mark.parametrize("dense", [True, False])
@pytest.mark.parametrize("seed", [61, 62])
def test_verify_mass_path_with_heavy_ties(port, dense, seed):
    """Integer-valued target rows (tens of thousands of equal keys per value) with top_k = 0 or
    above the list limit: the p of each draft, the residual draw that leaves the draft out (the
    one-hot case: an excluded composite inside a bin that must be refined by key digits) and the
    dense residual over all ids run on the mass path, against the oracle bit for bit."""
    streams, k = 12, 4
    d = W.config4(streams=streams, k=k, seed=seed, stochastic=True, masked=True)
    rng = np.random.default_rng(seed + 1000)
    tgt = W.bf16_bits_to_f32(d["target_bits"])
    tgt = np.clip(np.rint(tgt / 1.5), -4, 4).astype(np.float32)
    for s in range(streams):  # drafts on a well-populated value, on the top value, or far above it
        for i in range(k):
            tgt[s * (k + 1) + i, d["drafts"][s, i]] = float(rng.choice([2.0, 4.0, 16.0]))
    d["target_bits"] = W.f32_to_bf16_bits(tgt)
    p = d["params"]
    p["top_k"] = rng.choice(np.array([0, 0, 300, 1000, 40], np.int32), size=streams)
    p["top_p"] = rng.choice(np.array([1.0, 0.95, 0.8], np.float32), size=streams)
    p["temperature"] = rng.choice(np.array([0.5, 1.0, 2.0], np.float32), size=streams)
    p["min_p"] = np.where(rng.random(streams) < 0.25, np.float32(0.01), np.float32(0.0))
    g = check(port, d, dense)
    assert (g["status"] == 0).all()
    assert g["accepted"].min() < k  # some rejections, so residual draws run


def test_verify_extreme_parameters(port):
    """Temperatures of 1e-3 and 1,000, top_p at its limits, drafts whose q is exactly zero (the
    accept ratio's 1e-12 floor) or one, and uniforms at the ends of the unit interval."""
    streams, k = 12, 4
    d = W.config4(streams=streams, k=k, seed=81, stochastic=True, masked=False)
    rng = np.random.default_rng(82)
    p = d["params"]
    p["temperature"] = rng.choice(np.array([1e-3, 0.05, 20.0, 1000.0], np.float32), size=streams)
    p["top_k"] = rng.choice(np.array([0, 1, 257, 40], np.int32), size=streams)
    p["top_p"] = rng.choice(np.array([1.0, 0.999999, 1e-6], np.float32), size=streams)
    q = d["q"].reshape(streams, k, -1)
    for s in range(0, streams, 3):
        q[s, 0, d["drafts"][s, 0]] = 0.0  # a draft the drafter gave no mass
    for s in range(1, streams, 3):
        q[s, 1] = 0.0
        q[s, 1, d["drafts"][s, 1]] = 1.0  # a one-hot draft distribution, stored densely
    d["q"] = q.reshape(streams * k, -1)
    u = d["uniforms"]
    u[:3, 0] = [0.0, 1.0 - 2.0 ** -53, 1e-12]
    for dense in (True, False):
        g = check(port, d, dense)
        assert (g["status"] == 0).all()
