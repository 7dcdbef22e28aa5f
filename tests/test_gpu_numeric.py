"""GPU parity of sixi_smp_numeric_policy (NaN / Inf inspection and policy, in place) against the
CPU oracle (orc_numeric_policy, pinned to the engine's inspect_and_apply_numeric_policy by
tests/test_numeric.py): every report field and every rewritten logit bit for bit, for both
policies, aligned and unaligned rows, and vocabularies that take 1 to 8 CTAs per row."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import has_gpu
from oracle import binding as B

pytestmark = pytest.mark.gpu

if not has_gpu():
    pytest.skip("no CUDA device", allow_module_level=True)

import torch  # noqa: E402

import sixi_smp as S  # noqa: E402
from sixi_smp import workloads as W  # noqa: E402

DEV = torch.device("cuda:0")
FIELDS = ("healthy", "request_corrupted", "state_invalidated", "emergency_clamped", "status", "nan_count",
          "inf_count", "first_bad_index")


def make_rows(rng, rows, vocab):
    x = rng.normal(0.0, 40.0, size=(rows, vocab)).astype(np.float32)
    for r in range(rows):
        kind = r % 4
        if kind == 0:
            continue  # finite row
        k = int(rng.integers(1, 40))
        idx = rng.choice(vocab, size=min(k, vocab), replace=False)
        x[r, idx] = rng.choice(np.array([np.nan, np.inf, -np.inf], np.float32), size=idx.size)
        if kind == 3:
            x[r, vocab - 1] = np.nan  # the last element of the last CTA of the row
    return x


def check(rows_host, stride, vocab, policy, clamp, offset=0):
    """Runs the device pass on rows laid out with `stride` (and `offset` elements before row 0),
    then compares with the oracle row by row."""
    n = rows_host.shape[0]
    buf = np.full(offset + n * stride, 7.0, np.float32)
    for r in range(n):
        buf[offset + r * stride: offset + r * stride + vocab] = rows_host[r]
    d = torch.from_numpy(buf).to(DEV)
    view = d[offset:].as_strided((n, vocab), (stride, 1))
    smp = S.Sampler(0, max(n, 1), vocab)
    rep = S.numeric_reports(smp.numeric_policy(view, policy, clamp))
    torch.cuda.synchronize()
    got = d.cpu().numpy()
    smp.close()
    o = B.port()
    for r in range(n):
        want = rows_host[r].copy()
        st, wr = o.numeric_policy(want, policy, clamp)
        for f in FIELDS:
            assert rep[r][f] == wr[f], (r, f, rep[r][f], wr[f])
        row = got[offset + r * stride: offset + r * stride + vocab]
        assert row.view(np.uint32).tolist() == want.view(np.uint32).tolist(), r
        if r + 1 < n:  # the padding between rows is untouched
            pad = got[offset + r * stride + vocab: offset + (r + 1) * stride]
            assert (pad == 7.0).all(), r
    return rep


@pytest.mark.parametrize("policy", [S.NUMERIC_FAIL, S.NUMERIC_CLAMP])
@pytest.mark.parametrize("clamp", [100.0, 0.0, -25.0])
def test_full_vocab_rows(policy, clamp):
    rng = np.random.default_rng(int(10 * policy + abs(clamp)))
    vocab = W.QWEN_VOCAB
    x = make_rows(rng, 16, vocab)
    rep = check(x, vocab, vocab, policy, clamp)
    assert rep["healthy"].tolist() == [1 if r % 4 == 0 else 0 for r in range(16)]


@pytest.mark.parametrize("vocab", [1, 33, 4097, 8193, 200_003])
def test_vocab_sizes_and_unaligned_rows(vocab):
    """1 to 8 CTAs per row; a stride that is a multiple of 4 takes the 16-byte path (with a ragged
    tail for these odd vocabularies); odd strides and a 4-byte offset take the scalar path."""
    rng = np.random.default_rng(vocab)
    x = make_rows(rng, 6, vocab)
    for policy in (S.NUMERIC_FAIL, S.NUMERIC_CLAMP):
        check(x, vocab, vocab, policy, 50.0)
        check(x, vocab + (-vocab) % 4 + 4, vocab, policy, 50.0)
        check(x, vocab + 1, vocab, policy, 50.0, offset=1)
        check(x, vocab + 4, vocab, policy, 0.0, offset=4)


def test_large_batch_one_cta_per_row():
    """A batch that fills the GPU by itself runs one CTA per row (no cluster, 16-byte loads)."""
    rng = np.random.default_rng(77)
    vocab = W.QWEN_VOCAB
    x = make_rows(rng, 320, vocab)
    for policy in (S.NUMERIC_FAIL, S.NUMERIC_CLAMP):
        check(x, vocab, vocab, policy, 60.0)


def test_engine_unit_vectors_on_device():
    """The engine's own test rows (test_routing_and_numerics.cpp:415-460), one per policy."""
    rows = np.array([[1.0, 2.5, np.nan, -3.0, np.inf], [1.0, np.nan, np.inf, -np.inf, 500.0]], np.float32)
    rep = check(rows[:1], 5, 5, S.NUMERIC_FAIL, 100.0)
    assert rep[0]["status"] == 16 and rep[0]["first_bad_index"] == 2
    rep = check(rows[1:], 5, 5, S.NUMERIC_CLAMP, 100.0)
    assert rep[0]["emergency_clamped"] == 1 and rep[0]["inf_count"] == 2


def test_clamp_then_sample_matches_oracle(port):
    """The engine's order: policy on the logits, then sampling of the clamped rows."""
    from test_gpu_parity import check_against_oracle, run_sample

    rng = np.random.default_rng(3)
    d = W.config2(rows=16, seed=5)
    x = d["logits"]
    x[1, 17] = np.nan
    x[2, 900] = np.inf
    x[3, 4] = -np.inf
    t = torch.from_numpy(x.copy()).to(DEV)
    smp = S.Sampler(0, 16, x.shape[1])
    smp.numeric_policy(t, S.NUMERIC_CLAMP, 30.0)
    torch.cuda.synchronize()
    clamped = t.cpu().numpy()
    smp.close()
    want = x.copy()
    for r in range(16):
        B.port().numeric_policy(want[r], S.NUMERIC_CLAMP, 30.0)
    assert clamped.view(np.uint32).tolist() == want.view(np.uint32).tolist()
    d["logits"] = clamped
    u = rng.random(16)
    tok, st = run_sample(d, u)
    assert (st == 0).all()
    check_against_oracle(port, d, u, tok, st)
