"""json_schema grammar masks on the device (include/sixi_schema.h) over a 151,936-token synthetic
BPE-like vocabulary, against the library's host automaton (sixi_schema_check_text, whose grammar
tests/test_json_schema.py pins to an independent validator):

  masks        for rows at prefixes of valid documents, bit i is set exactly when the host accepts
               the prefix followed by token i (end-of-sequence: when the prefix is complete), except
               that the device never allows a token opening more than SIXI_SCHEMA_MASK_OPENS
               containers at once
  advance      token sequences applied on the device: rows that stay prefixes report OK, the first
               refused token freezes the row with SIXI_INVALID_ARGUMENT
  decoding     fill_masks -> sixi_smp_sample (masked) -> advance until end-of-sequence: every
               finished answer is a document the independent validator accepts
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import has_gpu

pytestmark = pytest.mark.gpu

if not has_gpu():
    pytest.skip("no CUDA device", allow_module_level=True)

import torch  # noqa: E402

from oracle.schema_oracle import Validator  # noqa: E402
from sixi_smp.json_grammar import Tokenizer, json_vocab  # noqa: E402
from sixi_smp.json_schema import COMPLETE, NOT_PREFIX, SchemaGrammar  # noqa: E402
from test_json_schema import SCHEMAS, docs  # noqa: E402

V = 151_936
OPENS = 6  # SIXI_SCHEMA_MASK_OPENS


@pytest.fixture(scope="module")
def vocab():
    toks, flags, eos = json_vocab(V, seed=5)
    return toks, flags, eos, Tokenizer(toks, flags)


def prefix_rows(name, tk, rows, seed):
    rng = np.random.default_rng(seed)
    ds = docs(name, rows, seed)
    seqs = []
    for d in ds:
        ids = tk.encode(d)
        seqs.append(ids[:int(rng.integers(0, len(ids) + 1))])
    L = max(1, max(len(s) for s in seqs))
    out = np.zeros((rows, L), np.int32)
    lens = np.array([len(s) for s in seqs], np.int32)
    for r, s in enumerate(seqs):
        out[r, :len(s)] = s
    return out, lens, seqs


@pytest.mark.parametrize("name", ["person", "tree", "formats", "enum"])
def test_masks_match_the_host_automaton(vocab, name):
    toks, flags, eos, tk = vocab
    g = SchemaGrammar(0, SCHEMAS[name], toks, flags, eos)
    rows = 6
    pre, lens, seqs = prefix_rows(name, tk, rows, seed=3 + len(name))
    st = g.new_states(rows)
    ast = g.advance(st, torch.from_numpy(pre).cuda(), torch.from_numpy(lens).cuda())
    assert (ast.cpu().numpy() == 0).all()
    masks = g.fill_masks(st)
    torch.cuda.synchronize()
    got = masks.cpu().numpy().view(np.uint32)
    bits = np.unpackbits(got.view(np.uint8).reshape(rows, -1), axis=1, bitorder="little")[:, :V].astype(bool)
    for r in range(rows):
        text = b"".join(toks[i] for i in seqs[r])
        base = g.check_text(text)
        assert base != NOT_PREFIX
        want = np.zeros(V, bool)
        for i, t in enumerate(toks):
            if i == eos:
                want[i] = base == COMPLETE
            elif t and not flags[i] & 1:
                want[i] = g.check_text(text + t) != NOT_PREFIX
        extra = bits[r] & ~want
        assert not extra.any(), (r, [toks[i] for i in np.nonzero(extra)[0][:5]])
        missing = np.nonzero(want & ~bits[r])[0]
        for i in missing:  # only tokens opening more containers than the mask walk holds
            assert toks[i].count(b"{") + toks[i].count(b"[") >= OPENS, (r, text, toks[i])
        assert want.sum() > 0
    g.close()


def test_advance_refuses_like_the_host(vocab):
    toks, flags, eos, tk = vocab
    g = SchemaGrammar(0, SCHEMAS["person"], toks, flags, eos)
    rows = 24
    rng = np.random.default_rng(11)
    pre, lens, seqs = prefix_rows("person", tk, rows, seed=12)
    # replace one token of half the rows with a random one: often refused
    for r in range(0, rows, 2):
        if lens[r] > 0:
            pre[r, int(rng.integers(0, lens[r]))] = int(rng.integers(0, V))
    st = g.new_states(rows)
    ast = g.advance(st, torch.from_numpy(pre).cuda(), torch.from_numpy(lens).cuda()).cpu().numpy()
    for r in range(rows):
        ids = [int(x) for x in pre[r, :lens[r]]]
        ok = True
        text = b""
        for i in ids:
            if i == eos or (flags[i] & 1) or not toks[i] or g.check_text(text + toks[i]) == NOT_PREFIX:
                ok = False
                break
            text += toks[i]
        assert (ast[r] == 0) == ok, (r, ast[r], ok)
    g.close()


def test_constrained_decoding_produces_valid_documents(vocab):
    import sixi_smp as S

    toks, flags, eos, _ = vocab
    rows, steps = 16, 300
    # closed schemas (every key typed is a declared one), so that random sampling finishes; open
    # objects with required keys (allof) rarely do, and their merging is a compile-time step the
    # host tests cover
    for name in ("person", "tuple", "formats"):
        g = SchemaGrammar(0, SCHEMAS[name], toks, flags, eos)
        v = Validator(SCHEMAS[name])
        bias = torch.tensor([2.0 * (b'"' in t) + 4.0 * (b"}" in t or b"]" in t) for t in toks], device="cuda")
        bias[eos] = 6.0
        gen = torch.Generator(device="cuda")
        gen.manual_seed(21)
        smp = S.Sampler(0, rows, V)
        params = S.make_params(rows, temperature=np.where(np.arange(rows) % 4 == 0, 0.0, 0.9), top_k=0, top_p=0.95,
                               flags=S.ROW_MASKED, seed=np.arange(rows, dtype=np.uint64) + 5)
        d_params = torch.from_numpy(params.view(np.uint8)).cuda()
        st = g.new_states(rows)
        masks = torch.empty((rows, (V + 31) // 32), dtype=torch.int32, device="cuda")
        out = [[] for _ in range(rows)]
        ended = np.zeros(rows, bool)
        for step in range(steps):
            logits = torch.randn((rows, V), generator=gen, device="cuda") * 2.0 + bias
            g.fill_masks(st, out=masks)
            tok, sts = smp.sample(logits, d_params, masks=masks, step=step)
            ast = g.advance(st, tok)
            tok, sts, ast = tok.cpu().numpy(), sts.cpu().numpy(), ast.cpu().numpy()
            for r in range(rows):
                if ended[r]:
                    continue  # a finished row has an empty mask: its sampler status is an error
                assert sts[r] == 0 and ast[r] == 0, (name, step, r, sts[r], ast[r])
                if tok[r] == eos:
                    ended[r] = True
                else:
                    out[r].append(int(tok[r]))
            if ended.all():
                break
        smp.close()
        for r in range(rows):
            text = b"".join(toks[i] for i in out[r])
            if ended[r]:
                assert v.accepts(text), (name, text)
            else:
                assert g.check_text(text) != NOT_PREFIX
        assert ended.sum() >= rows // 2, (name, ended.sum())
        g.close()


def test_malformed_states_are_frozen_not_walked(vocab):
    toks, flags, eos, tk = vocab
    g = SchemaGrammar(0, SCHEMAS["person"], toks, flags, eos)
    st = g.new_states(4)
    raw = st.cpu().numpy().copy()
    words = raw.view(np.uint32)  # [4, 200]: depth, failed, pad[6], then 24-byte frames
    words[1, 0] = 40             # deeper than SIXI_SCHEMA_MAX_DEPTH
    words[2, 8] = 1_000_000      # the root frame's node past the program
    words[3, 0] = 2              # a second frame of kind F_ROOT: only the bottom frame is a root
    st.copy_(torch.from_numpy(raw))
    masks = g.fill_masks(st).cpu().numpy()
    assert masks[0].any() and not masks[1:].any()
    tok = torch.tensor([tk.encode(b"{")[0]] * 4, dtype=torch.int32, device="cuda")
    ast = g.advance(st, tok).cpu().numpy()
    assert ast[0] == 0 and (ast[1:] != 0).all(), ast
    g.close()


def test_large_batches_give_the_same_masks(vocab):
    # 640 rows: one block per row, whose walk queue fills and is walked several times in the
    # middle of the row; against the same states masked four rows at a time
    toks, flags, eos, tk = vocab
    for name in ("person", "formats"):
        g = SchemaGrammar(0, SCHEMAS[name], toks, flags, eos)
        pre, lens, _ = prefix_rows(name, tk, 64, seed=41)
        st = g.new_states(64)
        assert (g.advance(st, torch.from_numpy(pre).cuda(), torch.from_numpy(lens).cuda()).cpu().numpy() == 0).all()
        big = st.repeat(10, 1)
        m_big = g.fill_masks(big)
        m_small = torch.cat([g.fill_masks(big[i:i + 4]) for i in range(0, big.shape[0], 4)])
        torch.cuda.synchronize()
        assert torch.equal(m_big, m_small), name
        g.close()
