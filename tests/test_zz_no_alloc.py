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


def _call_static(vocab, target, drafts, params, outs, draft_probs=None, uniforms=None, device=0):
    """sixi_smp_verify_static through the C ABI with caller-owned outputs (nothing allocated here)."""
    import ctypes

    S_, k = drafts.shape
    rows = S.Sampler._rows(target)
    ptr = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return S._lib().sixi_smp_verify_static(device, vocab, ctypes.byref(rows), ptr(draft_probs), ptr(drafts), None,
                                           S_, k, ptr(params), None, None, None, ptr(uniforms), 0,
                                           *[ptr(o) for o in outs], None)


def test_static_verify_warm_call_allocates_no_device_memory():
    """A warm call (after the first one on the device) changes nothing in the device's free memory:
    the workspace is the static array and the caller owns inputs and outputs."""
    vocab = 4097
    d = W.config4(streams=8, k=8, vocab=vocab, seed=31, stochastic=True, masked=False)
    target, drafts, params = dev(d["target_bits"]), dev(d["drafts"]), dev(d["params"])
    q, u = dev(d["q"]), dev(d["uniforms"])
    outs = [torch.empty(8, dtype=torch.int32, device=DEV), torch.empty((8, 9), dtype=torch.int32, device=DEV)] + \
        [torch.empty(8, dtype=torch.int32, device=DEV) for _ in range(4)]
    assert _call_static(vocab, target, drafts, params, outs, q, u) == 0  # first call: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(DEV)
    for _ in range(3):
        assert _call_static(vocab, target, drafts, params, outs, q, u) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(DEV)
    assert free1 == free0, (free0, free1)
    smp = S.Sampler(0, 128, vocab)
    ref = smp.verify(target, drafts, params, draft_probs=q, uniforms=u)
    torch.cuda.synchronize()
    for k_, o in zip(KEYS, outs):
        assert np.array_equal(ref[k_].cpu().numpy(), o.cpu().numpy()), k_
    smp.close()


def test_static_verify_on_another_device_restores_the_current_one():
    """With two GPUs: a call for device 1 while device 0 is current runs on device 1 (its own
    workspace address) and leaves device 0 current."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    vocab = 4097
    d1 = torch.device("cuda:1")
    x = W.config4(streams=4, k=8, vocab=vocab, seed=41, stochastic=True, masked=False)

    def on(a, dv):
        t = dev(a)
        return None if t is None else t.to(dv)

    target, drafts, params, q, u = (on(x[n], d1) for n in ("target_bits", "drafts", "params", "q", "uniforms"))
    outs = [torch.empty(4, dtype=torch.int32, device=d1), torch.empty((4, 9), dtype=torch.int32, device=d1)] + \
        [torch.empty(4, dtype=torch.int32, device=d1) for _ in range(4)]
    torch.cuda.set_device(0)
    assert _call_static(vocab, target, drafts, params, outs, q, u, device=1) == 0
    assert torch.cuda.current_device() == 0
    torch.cuda.synchronize(d1)
    smp = S.Sampler(1, 64, vocab)
    ref = smp.verify(target, drafts, params, draft_probs=q, uniforms=u)
    torch.cuda.synchronize(d1)
    for k_, o in zip(KEYS, outs):
        assert np.array_equal(ref[k_].cpu().numpy(), o.cpu().numpy()), k_
    smp.close()
