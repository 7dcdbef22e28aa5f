"""sixi_smp_verify_static (no handle, no allocation, static device workspace) against the
handle-based sixi_smp_verify on the same inputs.

Collected last (file name) so that it runs both alone and after every other GPU test of the session;
it makes several calls in a row, so the shared static workspace is reused between them.
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

DEV = torch.device("cuda:0")
KEYS = ("accepted", "tokens", "n_tokens", "first_reject", "uniforms_used", "status")


def dev(a):
    if a is None:
        return None
    if a.dtype.names is not None:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.uint8)).to(DEV)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(DEV)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(DEV).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def both(smp, vocab, d, dense, uniforms=True, n_drafts=None):
    kw = dict(draft_probs=dev(d["q"]) if dense else None, n_drafts=dev(n_drafts), masks=dev(d["masks"]),
              hist=dev(d["hist"]), hist_off=dev(d["hist_off"]), uniforms=dev(d["uniforms"]) if uniforms else None,
              step=3)
    target, drafts, params = dev(d["target_bits"]), dev(d["drafts"]), dev(d["params"])
    ref = smp.verify(target, drafts, params, **kw)
    got = S.verify_static(vocab, target, drafts, params, **kw)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in ref.items()}, {k: v.cpu().numpy() for k, v in got.items()}


def assert_same(ref, got):
    for k in KEYS:
        assert np.array_equal(ref[k], got[k]), (k, ref[k], got[k])


def test_static_verify_calls_in_a_row_small_vocab():
    vocab = 4097
    smp = S.Sampler(0, 256, vocab)
    seen = []
    for seed, dense in [(11, True), (12, False), (11, True)]:  # the third call repeats the first
        d = W.config4(streams=6, k=4, vocab=vocab, seed=seed, stochastic=True, masked=True)
        ref, got = both(smp, vocab, d, dense)
        assert_same(ref, got)
        seen.append(got)
    assert_same(seen[0], seen[2])
    d = W.config4(streams=5, k=3, vocab=vocab, seed=13, stochastic=False, masked=False)
    ref, got = both(smp, vocab, d, True, uniforms=False, n_drafts=np.array([3, 0, 1, 2, 3], np.int32))
    assert_same(ref, got)
    smp.close()


def test_static_verify_full_vocab():
    vocab = W.QWEN_VOCAB
    smp = S.Sampler(0, 128, vocab)
    for seed, dense in [(21, True), (22, False)]:
        d = W.config4(streams=8, k=8, vocab=vocab, seed=seed, stochastic=True, masked=True)
        ref, got = both(smp, vocab, d, dense)
        assert_same(ref, got)
    smp.close()


def test_static_verify_rejects_more_rows_than_the_workspace():
    vocab = 64
    k = 7
    streams = S.STATIC_VERIFY_ROWS // (k + 1) + 1  # one stream past the static workspace
    target = torch.zeros((streams * (k + 1), vocab), dtype=torch.float32, device=DEV)
    drafts = torch.zeros((streams, k), dtype=torch.int32, device=DEV)
    params = dev(S.make_params(streams, temperature=0.0))
    with pytest.raises(S.SixiError) as ei:
        S.verify_static(vocab, target, drafts, params)
    assert ei.value.status == 2  # SIXI_OUT_OF_BOUNDS
