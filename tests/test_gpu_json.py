"""Device parity of the JSON-object grammar-mask producer (include/sixi_json.h) against the CPU
automaton (oracle/sixi_json_oracle.c, itself pinned to Python's json module by test_json.py).

Masks, advanced states and per-draft states must be bit-identical to the oracle's over the full
151,936-token synthetic vocabulary; a constrained decoding loop through sixi_smp_sample must only
ever produce prefixes of JSON objects, and every finished answer must parse."""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import has_gpu
from oracle import binding as B

pytestmark = pytest.mark.gpu

V = 151_936


@pytest.fixture(scope="module")
def setup():
    if not has_gpu():
        pytest.skip("no GPU")
    import torch

    from sixi_smp.json_grammar import JsonGrammar, Tokenizer, json_documents, json_vocab

    toks, flags, eos = json_vocab(V, seed=5)
    g = JsonGrammar(0, toks, flags, eos)
    v = B.JsonVocab(toks, flags, eos)
    tk = Tokenizer(toks, flags)
    docs = json_documents(200, seed=21)
    yield dict(torch=torch, toks=toks, flags=flags, eos=eos, g=g, v=v, tk=tk, docs=docs)
    g.close()


def _states(s, rows, seed):
    from sixi_smp.json_grammar import prefix_states_tokens

    torch = s["torch"]
    pre, lens = prefix_states_tokens(s["docs"], s["tk"], rows, seed=seed)
    host = np.zeros((rows, 32), np.uint8)
    st = B.json_advance(B.port(), s["v"], host, pre, lens)
    assert (st == 0).all()
    dev = s["g"].new_states(rows)
    ost = s["g"].advance(dev, torch.from_numpy(pre).cuda(), torch.from_numpy(lens).cuda())
    torch.cuda.synchronize()
    assert (ost.cpu().numpy() == 0).all()
    assert (dev.cpu().numpy() == host).all(), "advanced states differ from the oracle's"
    return host, dev


@pytest.mark.parametrize("seed", [1, 2])
def test_masks_match_oracle(setup, seed):
    s = setup
    host, dev = _states(s, 64, seed)
    got = s["g"].fill_masks(dev).cpu().numpy().view(np.uint32)
    want = B.json_fill_masks(B.port(), s["v"], host, n_threads=8)
    assert got.shape == want.shape
    bad = np.nonzero((got != want).any(axis=1))[0]
    assert bad.size == 0, f"rows {bad[:8]} modes {host[bad[:8], 0]}"
    modes = set(host[:, 0].tolist())
    assert len(modes) >= 5, modes  # the prefixes cover several automaton modes


def test_special_states(setup):
    """Start, done, failed, deep nesting, split UTF-8 and escape states."""
    s = setup
    torch = s["torch"]
    o = B.port()
    texts = [b"", b"  ", b"{}", b'{"a":"\xe6\x97', b'{"a":"\\u00', b'{"a":' + b"[" * 127, b'{"a":tr', b'{"a":-',
             b'{"a":1.5e', b'{"a":"x\\', b'{"k":{"k":{"k":[1,', b'{"\xf0\x9f', b'{"a":0']
    host = np.zeros((len(texts) + 1, 32), np.uint8)
    for i, t in enumerate(texts):
        assert B.json_feed(o, host[i], t), t
    host[-1, 6] = 1  # a failed row: empty mask
    dev = torch.from_numpy(host).cuda()
    got = s["g"].fill_masks(dev).cpu().numpy().view(np.uint32)
    want = B.json_fill_masks(o, s["v"], host, n_threads=8)
    assert (got == want).all()
    assert not got[-1].any()
    eos = s["eos"]
    assert (got[2, eos // 32] >> (eos % 32)) & 1  # a complete document: end-of-sequence only
    assert int(np.unpackbits(got[2].view(np.uint8)).sum()) == 1


def test_advance_refusals_match_oracle(setup):
    s = setup
    torch = s["torch"]
    host, dev = _states(s, 48, 3)
    rng = np.random.default_rng(4)
    tok = rng.integers(-2, V + 2, size=48).astype(np.int32)
    tok[:8] = s["eos"]
    h2 = host.copy()
    want = B.json_advance(B.port(), s["v"], h2, tok)
    got = s["g"].advance(dev, torch.from_numpy(tok).cuda()).cpu().numpy()
    assert (got == want).all()
    assert (dev.cpu().numpy() == h2).all()
    assert (want == 1).any() and (want == 0).any()


def test_expand_drafts_match_oracle(setup):
    s = setup
    torch = s["torch"]
    host, dev = _states(s, 16, 5)
    k = 8
    drafts = np.zeros((16, k), np.int32)
    rng = np.random.default_rng(6)
    for r in range(16):  # mostly valid continuations (greedy on the oracle's masks), some random
        st = host[r].copy()
        for j in range(k):
            m = B.json_fill_masks(B.port(), s["v"], st[None])[0]
            allowed = np.nonzero(np.unpackbits(m.view(np.uint8), bitorder="little")[:V])[0]
            if allowed.size and rng.random() < 0.85:
                drafts[r, j] = int(rng.choice(allowed))
                if drafts[r, j] != s["eos"]:
                    B.json_feed(B.port(), st, s["toks"][drafts[r, j]])
            else:
                drafts[r, j] = int(rng.integers(0, V))
    nd = rng.integers(0, k + 1, size=16).astype(np.int32)
    want = B.json_expand(B.port(), s["v"], host, drafts, nd)
    got = s["g"].expand_drafts(dev, torch.from_numpy(drafts).cuda(), torch.from_numpy(nd).cuda())
    assert (got.cpu().numpy() == want).all()
    masks = s["g"].fill_masks(got).cpu().numpy().view(np.uint32)
    assert (masks == B.json_fill_masks(B.port(), s["v"], want, n_threads=8)).all()


def test_constrained_decoding_produces_json_objects(setup):
    """fill_masks -> sixi_smp_sample (masked rows) -> advance, on device, until the answers end."""
    import sixi_smp as S
    from sixi_smp.json_grammar import DONE

    s = setup
    torch = s["torch"]
    rows, steps = 16, 400
    toks = s["toks"]
    # random logits with a pull towards closing strings and containers, so that answers end
    bias = torch.tensor([3.0 * (b'"' in t) + 5.0 * (b"}" in t or b"]" in t) for t in toks], device="cuda")
    gen = torch.Generator(device="cuda")
    gen.manual_seed(8)
    smp = S.Sampler(0, rows, V)
    params = S.make_params(rows, temperature=np.where(np.arange(rows) % 4 == 0, 0.0, 0.9), top_k=0, top_p=0.95,
                           flags=S.ROW_MASKED, seed=np.arange(rows, dtype=np.uint64) + 77)
    d_params = torch.from_numpy(params.view(np.uint8)).cuda()
    states = s["g"].new_states(rows)
    masks = torch.empty((rows, (V + 31) // 32), dtype=torch.int32, device="cuda")
    out = [[] for _ in range(rows)]
    for step in range(steps):
        logits = torch.randn((rows, V), generator=gen, device="cuda") * 2.0 + bias
        s["g"].fill_masks(states, out=masks)
        tok, st = smp.sample(logits, d_params, masks=masks, step=step)
        ast = s["g"].advance(states, tok)
        tok, st, ast = tok.cpu().numpy(), st.cpu().numpy(), ast.cpu().numpy()
        assert (st == 0).all() and (ast == 0).all(), (step, st, ast)
        for r in range(rows):
            if tok[r] != s["eos"]:
                out[r].append(int(tok[r]))
        if (states.cpu().numpy()[:, 0] == DONE).all():
            break
    smp.close()
    fin = states.cpu().numpy()
    done = 0
    for r in range(rows):
        text = b"".join(toks[i] for i in out[r])
        if fin[r, 0] == DONE:
            assert isinstance(json.loads(text.decode("utf-8")), dict), text
            done += 1
        else:
            chk = np.zeros(32, np.uint8)
            assert B.json_feed(B.port(), chk, text) and (chk == fin[r]).all()
    assert done >= rows // 2, done


def test_speculative_step_with_grammar_masks(setup):
    """expand_drafts -> fill_masks -> sixi_smp_verify (masked target rows) -> advance by the
    committed tokens: a drafted token that breaks the grammar is rejected at its position, and
    every committed token keeps the answer a JSON prefix (the oracle checks each)."""
    import sixi_smp as S

    s = setup
    torch = s["torch"]
    rows_s, k = 8, 4
    host, dev = _states(s, rows_s, 9)
    rng = np.random.default_rng(10)
    o = B.port()
    drafts = np.zeros((rows_s, k), np.int32)
    bad_at = np.full(rows_s, -1)
    for r in range(rows_s):
        st = host[r].copy()
        for j in range(k):
            m = B.json_fill_masks(o, s["v"], st[None])[0]
            allowed = np.nonzero(np.unpackbits(m.view(np.uint8), bitorder="little")[:V])[0]
            if r % 2 == 1 and j == 2 and bad_at[r] < 0:  # a draft the grammar refuses
                refused = np.setdiff1d(np.arange(V), allowed)
                drafts[r, j] = int(rng.choice(refused))
                bad_at[r] = j
            elif bad_at[r] < 0:
                drafts[r, j] = int(rng.choice(allowed))
                if drafts[r, j] != s["eos"]:
                    B.json_feed(o, st, s["toks"][drafts[r, j]])
            else:
                drafts[r, j] = int(rng.integers(0, V))
    d_drafts = torch.from_numpy(drafts).cuda()
    row_states = s["g"].expand_drafts(dev, d_drafts)
    masks = s["g"].fill_masks(row_states)
    # target logits that favour each draft strongly, so that only the grammar rejects
    tgt = torch.randn((rows_s * (k + 1), V), device="cuda")
    for r in range(rows_s):
        for j in range(k):
            tgt[r * (k + 1) + j, int(drafts[r, j])] += 30.0
    params = S.make_params(rows_s, temperature=0.0, flags=S.ROW_MASKED)
    smp = S.Sampler(0, rows_s * (k + 1), V)
    out = smp.verify(tgt, d_drafts, torch.from_numpy(params.view(np.uint8)).cuda(), masks=masks)
    acc = out["accepted"].cpu().numpy()
    ntok = out["n_tokens"].cpu().numpy()
    toks = out["tokens"].cpu().numpy()
    assert (out["status"].cpu().numpy() == 0).all()
    for r in range(rows_s):
        if bad_at[r] >= 0:
            assert acc[r] <= bad_at[r], (r, acc[r], bad_at[r])
    # commit and advance; the oracle must accept every committed token
    st = s["g"].advance(dev, out["tokens"], n_tokens=out["n_tokens"])
    assert (st.cpu().numpy() == 0).all()
    for r in range(rows_s):
        chk = host[r].copy()
        for j in range(ntok[r]):
            if toks[r, j] != s["eos"]:
                assert B.json_feed(o, chk, s["toks"][toks[r, j]]), (r, j)
        assert (chk[:6] == dev.cpu().numpy()[r, :6]).all()
    smp.close()
