"""GPU parity of sixi_smp_suffix_draft (batched suffix n-gram drafting) against the CPU oracle
(orc_suffix_draft, pinned to the engine's SuffixDrafter by tests/test_suffix.py): match lengths
and drafts of every stream must be identical, for propose and propose_anchored, with staged and
unstaged windows."""

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
from test_suffix import histories  # noqa: E402

DEV = torch.device("cuda:0")


def run(hs, k, min_match, window, anchors=None):
    off = np.zeros(len(hs) + 1, np.int64)
    off[1:] = np.cumsum([h.size for h in hs])
    flat = np.concatenate(hs).astype(np.int32) if off[-1] else np.zeros(1, np.int32)
    smp = S.Sampler(0, 1, 64)
    a = None if anchors is None else torch.from_numpy(np.asarray(anchors, np.int32)).to(DEV)
    d, m = smp.suffix_draft(torch.from_numpy(flat).to(DEV), torch.from_numpy(off).to(DEV), k=k,
                            min_match_len=min_match, max_window_tokens=window, anchors=a)
    torch.cuda.synchronize()
    smp.close()
    return d.cpu().numpy(), m.cpu().numpy()


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_batches_match_oracle(seed):
    rng = np.random.default_rng(seed)
    hs = histories(rng, 48)
    o = B.port()
    found = 0
    for min_match, window, k in [(3, 16384, 8), (1, 100, 5), (2, 8, 1), (4, 16384, 33), (17, 16384, 4),
                                 (3, 40000, 8), (0, 16384, 8), (3, 16384, 0)]:
        for anchored in (False, True):
            anchors = [int(h[-1]) if h.size and i % 3 else int(rng.integers(0, 64)) for i, h in enumerate(hs)] \
                if anchored else None
            d, m = run(hs, k, min_match, window, anchors)
            for s, h in enumerate(hs):
                om, od = o.suffix_draft(h, min_match, window, k, None if anchors is None else anchors[s])
                assert m[s] == om, (seed, min_match, window, k, anchored, s, h.size, m[s], om)
                assert np.array_equal(d[s], od), (seed, min_match, window, k, anchored, s)
                found += om > 0
    assert found > 50


def test_engine_default_window_long_histories():
    """SuffixDrafter(3, 16384) on 20,000-token histories: the window and the 16 tokens below it are
    staged; random histories fall through to the exact-tail search."""
    rng = np.random.default_rng(9)
    hs = []
    for i in range(32):
        h = rng.integers(0, 151_936 if i % 2 else 50, size=20_000).astype(np.int32)
        if i % 4 == 1:
            h[5000:5012] = h[-12:]
        hs.append(h)
    d, m = run(hs, 8, 3, 16384)
    o = B.port()
    for s, h in enumerate(hs):
        om, od = o.suffix_draft(h, 3, 16384, 8)
        assert m[s] == om and np.array_equal(d[s], od), (s, m[s], om)
    assert (m[1::4] > 0).all()
