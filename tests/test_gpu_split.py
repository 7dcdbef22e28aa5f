"""The small-batch latency path of sixi_smp_sample (batches of at most 4 rows): greedy rows and rows
with 1 <= top_k <= 64 run as 16 vocabulary slices per row plus the merge, the batch's other rows on
the cluster path on a second stream. Checked against the CPU oracle, and against the cluster path
alone on the same inputs (sixi_smp_set_split_rows(0)): statuses equal, tokens equal except rows the
oracle comparison excuses at a CDF boundary.
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
from test_gpu_parity import check_against_oracle, dev, rand_small_case  # noqa: E402


def run(smp, d, u, step=0):
    tok, st = smp.sample(dev(d["logits"]), dev(d["params"]), masks=dev(d.get("masks")), hist=dev(d.get("hist")),
                         hist_off=dev(d.get("hist_off")) if d.get("hist") is not None else None,
                         uniforms=dev(u), step=step)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), st.cpu().numpy()


def both_paths(port, d, u, step=0):
    vocab = d.get("vocab", d["logits"].shape[1])
    smp = S.Sampler(0, 64, vocab)
    tok, st = run(smp, d, u, step)
    smp.set_split_rows(0)
    tok0, st0 = run(smp, d, u, step)
    smp.close()
    assert np.array_equal(st, st0), (st, st0)
    check_against_oracle(port, d, u, tok, st, step=step)
    check_against_oracle(port, d, u, tok0, st0, step=step)
    return tok, tok0


@pytest.mark.parametrize("vocab", [1, 33, 4097, 40000, 151_936])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_small_batches_random_params(port, vocab, dtype):
    rng = np.random.default_rng(vocab * 3 + (dtype == "bf16"))
    for rows in (1, 2, 3, 4):
        d = rand_small_case(rng, vocab, rows, dtype)
        u = rng.random(rows)
        both_paths(port, d, u)


def test_config1_rows_take_the_split_path(port):
    for greedy in (False, True):
        d = W.config1(greedy=greedy)
        for step in range(3):
            tok, tok0 = both_paths(port, d, None, step=step)
            assert np.array_equal(tok, tok0)


def test_mixed_batch_eligible_and_cluster_rows(port):
    # greedy, top_k 1 / 20 / 64 (split path) beside top_k 0 / 65 / 1000 (cluster path), penalties
    # with a long history, a frequency penalty past 16-bit counts (cluster path), masks
    vocab = 151_936
    rng = np.random.default_rng(9)
    for top_k in ([0, 20, 65, 1], [64, 0, 1000, 0], [20, 20, 20, 20]):
        rows = 4
        logits = rng.normal(0, 2.5, size=(rows, vocab)).astype(np.float32)
        W.boost_rows(rng, logits)
        t = np.array([0.7, 0.0, 1.1, 0.9], np.float32)
        params = S.make_params(rows, temperature=t, top_k=np.array(top_k, np.int32), top_p=0.9,
                               repetition_penalty=1.2, presence_penalty=0.3,
                               frequency_penalty=np.array([0.0, 0.2, 0.0, 0.1], np.float32), flags=S.ROW_MASKED)
        lens = np.array([64, 70_000, 3000, 8192])
        off = np.zeros(rows + 1, np.int64)
        off[1:] = np.cumsum(lens)
        hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int32)
        allowed = np.stack([W.run_mask(rng, vocab, f) for f in (0.6, 0.05, 1.0, 0.001)])
        d = dict(logits=logits, params=params, masks=W.pack_mask(allowed), hist=hist, hist_off=off, vocab=vocab)
        both_paths(port, d, rng.random(rows))


def test_split_path_inside_a_cuda_graph(port):
    d = W.config1()
    smp = S.Sampler(0, 4, d["logits"].shape[1])
    logits, params = dev(d["logits"]), dev(d["params"])
    hist, hoff = dev(d["hist"]), dev(d["hist_off"])
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    st = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        smp.sample(logits, params, hist=hist, hist_off=hoff, out_tokens=tok, out_status=st, step=0, stream=s)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for step in range(4):
            smp.sample(logits, params, hist=hist, hist_off=hoff, out_tokens=tok[0:1], out_status=st, step=step,
                       stream=s)
    g.replay()
    torch.cuda.synchronize()
    # the last captured step's token equals an eager call of that step
    t3, s3 = smp.sample(logits, params, hist=hist, hist_off=hoff, step=3)
    torch.cuda.synchronize()
    assert int(st[0]) == 0 and int(tok[0]) == int(t3[0]) and int(s3[0]) == 0
    del g
    smp.close()
