"""Vocab-sharded mode on one GPU: the rows are split into S vocabulary slices (views into the full
rows), stage 1 runs once per slice, the outputs are stacked rank-major as an all-gather would
leave them, and stage 2 merges them. Every row whose status is OK must draw the oracle's token
for the full row (exact except within 1e-6 of a CDF boundary); rows with top_k <= top_n must
always be OK; rows outside that guarantee may report SIXI_OUT_OF_BOUNDS.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import has_gpu, near_boundary

pytestmark = pytest.mark.gpu

if not has_gpu():
    pytest.skip("no CUDA device", allow_module_level=True)

import torch  # noqa: E402

import sixi_smp as S  # noqa: E402
from sixi_smp import workloads as W  # noqa: E402
from sixi_smp.sharded import ShardLayout  # noqa: E402
from test_gpu_parity import dev  # noqa: E402

OOB = 2  # SIXI_OUT_OF_BOUNDS


def run_sharded(smp, d, n_shards, top_n, uniforms, step=0):
    vocab = d["logits"].shape[1]
    lay = ShardLayout(vocab, n_shards)
    full = dev(d["logits"])
    params = dev(d["params"])
    masks = dev(d.get("masks"))
    hist = dev(d.get("hist"))
    hoff = dev(d.get("hist_off")) if d.get("hist") is not None else None
    cands, stats = [], []
    for r in range(n_shards):
        x = full[:, lay.offset(r):lay.offset(r) + lay.width(r)]
        c, s = smp.shard_candidates(x, lay.offset(r), lay.width(r), params, top_n=top_n, masks=masks, hist=hist,
                                    hist_off=hoff)
        cands.append(c)
        stats.append(s)
    tok, st = smp.merge_shards(torch.stack(cands), torch.stack(stats), params, uniforms=dev(uniforms), step=step)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), st.cpu().numpy()


def check(port, d, tok, st, uniforms, top_n, step=0):
    vocab = d["logits"].shape[1]
    p = d["params"]
    u = uniforms
    if u is None:
        u = np.array([port.philox_uniform(int(q["seed"]), int(q["counter"]) + step, 0) for q in p])
    otok, ost = port.sample_batch(d["logits"], p, d.get("masks"), d.get("hist"), d.get("hist_off"), u, step=step,
                                  vocab=vocab)
    n_oob = 0
    for r in range(len(tok)):
        if st[r] == OOB:
            k = int(p["top_k"][r])
            assert not (0 < k <= top_n) and p["temperature"][r] > 0, f"row {r}: top_k={k} must be exact"
            n_oob += 1
            continue
        assert st[r] == ost[r], (r, st[r], ost[r])
        if st[r] != 0 or tok[r] == otok[r]:
            continue
        h = None if d.get("hist") is None else d["hist"][d["hist_off"][r]:d["hist_off"][r + 1]]
        m = d["masks"][r] if d.get("masks") is not None and (p["flags"][r] & S.ROW_MASKED) else None
        assert near_boundary(port, d["logits"][r], p[r:r + 1], h, m, u[r]), (r, tok[r], otok[r])
    return n_oob


@pytest.mark.parametrize("n_shards", [2, 4, 8])
def test_sharded_config2_full_vocab(port, n_shards):
    d = W.config2(rows=32, seed=600 + n_shards)
    u = np.random.default_rng(n_shards).random(32)
    smp = S.Sampler(0, 64, d["logits"].shape[1])
    tok, st = run_sharded(smp, d, n_shards, 64, u)
    n_oob = check(port, d, tok, st, u, 64)
    assert n_oob <= int(np.sum(d["params"]["top_k"] == 0))  # only full-softmax rows may miss
    smp.close()


def test_sharded_top_k_rows_are_exact(port):
    """top_k <= top_n: every row exact, with masks, bf16, penalties and Philox uniforms."""
    rng = np.random.default_rng(7)
    d = W.config3(rows=24, seed=8)
    d["params"]["top_k"] = rng.choice(np.array([1, 5, 20, 40, 64], np.int32), size=24)
    d["params"]["temperature"] = np.where(d["params"]["temperature"] <= 0, 0.6, d["params"]["temperature"])
    smp = S.Sampler(0, 64, d["logits"].shape[1])
    for n_shards in (2, 3, 16):
        tok, st = run_sharded(smp, d, n_shards, 64, None, step=4)
        assert check(port, d, tok, st, None, 64, step=4) == 0
    bf = dict(d)
    bf["logits"] = W.f32_to_bf16_bits(d["logits"])
    tok, st = run_sharded(smp, bf, 4, 64, None, step=1)
    assert check(port, bf, tok, st, None, 64, step=1) == 0
    smp.close()


@pytest.mark.parametrize("vocab", [100, 4097, 40000])
def test_sharded_small_vocab_mixed(port, vocab):
    rng = np.random.default_rng(vocab)
    n = 16
    logits = rng.normal(0, 2.0, size=(n, vocab)).astype(np.float32)
    logits[:, ::7] = np.round(logits[:, ::7])  # ties
    params = S.make_params(n, temperature=rng.choice([0.0, 0.5, 1.0, 1.5], size=n).astype(np.float32),
                           top_k=rng.choice(np.array([0, 3, 16, 64, 200], np.int32), size=n),
                           top_p=rng.choice(np.array([1.0, 0.9, 0.3], np.float32), size=n),
                           min_p=rng.choice(np.array([0.0, 0.05], np.float32), size=n),
                           repetition_penalty=1.2, presence_penalty=0.3, frequency_penalty=0.1,
                           mode=S.ADAPTIVE)
    off = np.arange(n + 1, dtype=np.int64) * 40
    hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32)
    d = dict(logits=logits, params=params, hist=hist, hist_off=off, masks=None)
    u = rng.random(n)
    smp = S.Sampler(0, 64, vocab)
    for n_shards in (2, 5):
        tok, st = run_sharded(smp, d, n_shards, 32, u)
        check(port, d, tok, st, u, 32)
    smp.close()


def test_sharded_statuses(port):
    vocab = 3000
    n = 4
    logits = np.random.default_rng(1).normal(size=(n, vocab)).astype(np.float32)
    logits[1, 2999] = np.nan  # in the last shard
    params = S.make_params(n, temperature=0.8, top_k=10)
    masks = np.zeros((n, (vocab + 31) // 32), np.uint32)
    masks[:, :] = 0xFFFFFFFF
    masks[2, :] = 0  # nothing allowed
    params["flags"][2] = S.ROW_MASKED
    d = dict(logits=logits, params=params, masks=masks, hist=None, hist_off=None)
    u = np.full(n, 0.5)
    smp = S.Sampler(0, 8, vocab)
    tok, st = run_sharded(smp, d, 3, 16, u)
    assert st[1] == 16 and st[2] == 1 and st[0] == 0 and st[3] == 0
    check(port, d, tok, st, u, 16)
    smp.close()


@pytest.mark.parametrize("n_shards", [2, 8])
def test_sharded_heavy_ties_across_shards(port, n_shards):
    """Integer-valued rows: every shard's best top_n are equal keys, so the merge must order the
    gathered candidates by id across shards, exactly as the full row orders them."""
    rng = np.random.default_rng(900 + n_shards)
    vocab, n = W.QWEN_VOCAB, 16
    logits = rng.integers(-4, 5, size=(n, vocab)).astype(np.float32)
    logits[: n // 2] = np.minimum(logits[: n // 2], 2.0)  # half the rows: a third of the ids tie at the top
    params = S.make_params(n, temperature=rng.choice(np.array([0.0, 0.5, 1.0, 2.0], np.float32), size=n),
                           top_k=rng.choice(np.array([1, 5, 20, 64, 0], np.int32), size=n),
                           top_p=rng.choice(np.array([1.0, 0.9, 0.5], np.float32), size=n),
                           repetition_penalty=np.float32(1.2))
    lens = rng.integers(0, 1024, size=n)
    off = np.zeros(n + 1, dtype=np.int64)
    off[1:] = np.cumsum(lens)
    d = dict(logits=logits, params=params, masks=None, hist=rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32),
             hist_off=off)
    u = rng.random(n)
    smp = S.Sampler(0, 64, vocab)
    tok, st = run_sharded(smp, d, n_shards, 64, u)
    check(port, d, tok, st, u, 64)
    smp.close()
