"""The vocab-sharded step's collective plumbing on CPU ranks (gloo, world size 2): each rank holds
half of the vocabulary of every row, runs a host restatement of stage 1 on its slice, the
candidates and statistics are all-gathered by sixi_smp.sharded.sample_vocab_sharded, and each rank
merges them with a host stage 2 (the oracle applied to the merged candidates). Rows whose top_k
exceeds top_n (or is 0) cannot be certified from the candidates: the host stage 2 flags them
SIXI_OUT_OF_BOUNDS, and the second exchange round rebuilds their full rows from all ranks' slices
and samples them there. Both ranks must reach the oracle's tokens for every row.
"""

from __future__ import annotations

import socket
import struct

import numpy as np
import pytest

from conftest import REPO

N_ROWS, VOCAB, TOP_N = 12, 3001, 16


def _rows():
    import sys

    sys.path.insert(0, str(REPO / "sixi-asi_b200"))
    import sixi_smp as S

    rng = np.random.default_rng(5)
    logits = rng.normal(0, 2.0, size=(N_ROWS, VOCAB)).astype(np.float32)
    params = S.make_params(N_ROWS, temperature=rng.choice([0.0, 0.7, 1.3], size=N_ROWS).astype(np.float32),
                           top_k=rng.choice(np.array([1, 5, 16, 0, 40], np.int32), size=N_ROWS),
                           top_p=rng.choice(np.array([1.0, 0.8], np.float32), size=N_ROWS))
    u = rng.random(N_ROWS)
    return logits, params, u


def _stage1(x, off, width, params):
    import torch

    n = x.shape[0]
    cand = np.zeros((n, TOP_N, 2), np.int32)
    cand[:, :, 0] = np.float32(-np.inf).view(np.int32)
    cand[:, :, 1] = -1
    stats = np.zeros((n, 24), np.uint8)
    xs = x.numpy()
    for r in range(n):
        row = xs[r, :width]
        order = np.lexsort((np.arange(width), -row))[:TOP_N]  # logit desc, id asc
        cand[r, :len(order), 0] = row[order].view(np.int32)
        cand[r, :len(order), 1] = order + off
        t = float(params["temperature"][r])
        m = float(row.max())
        se = float(np.sum(np.exp((row.astype(np.float64) - m) / t))) if t > 0 else 0.0
        stats[r] = np.frombuffer(struct.pack("<fidii", m, width, se, 0, 0), np.uint8)
    return torch.from_numpy(cand), torch.from_numpy(stats)


def _stage2(g_cand, g_stats, params, u, port):
    import torch

    import sixi_smp as S
    from sixi_smp import workloads as W

    gc = g_cand.numpy()
    S_, n = gc.shape[0], gc.shape[1]
    tok = np.empty(n, np.int32)
    st = np.empty(n, np.int32)
    for r in range(n):
        row = np.zeros(VOCAB, np.float32)
        allowed = np.zeros(VOCAB, bool)
        for s in range(S_):
            for j in range(TOP_N):
                i = int(gc[s, r, j, 1])
                if i >= 0:
                    row[i] = gc[s, r, j, 0:1].view(np.float32)[0]
                    allowed[i] = True
        p = params[r:r + 1].copy()
        k = int(p["top_k"][0])
        if float(p["temperature"][0]) > 0 and (k == 0 or k > TOP_N):
            st[r], tok[r] = 2, -1  # the candidates cannot certify this row: second round
            continue
        p["flags"] = S.ROW_MASKED
        st[r], tok[r] = port.sample(row, p, None, W.pack_mask(allowed[None])[0], float(u[r]))
    return torch.from_numpy(tok), torch.from_numpy(st)


def _full_rows(full, rows, params, u, port):
    import torch

    rows = rows.numpy()
    tok, st = port.sample_batch(full.numpy(), params[rows], None, None, None, u[rows])
    return torch.from_numpy(tok), torch.from_numpy(st)


def _worker(rank: int, port_no: int, errq):
    import os
    import sys

    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "sixi-asi_b200"))
    import torch
    import torch.distributed as dist

    from oracle import binding
    from sixi_smp.sharded import ShardLayout, sample_vocab_sharded

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port_no)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        port = binding.port()
        logits, params, u = _rows()
        lay = ShardLayout(VOCAB, 2)
        mine = torch.from_numpy(np.ascontiguousarray(logits[:, lay.offset(rank):lay.offset(rank) + lay.width(rank)]))
        tok, st = sample_vocab_sharded(
            mine, lay, rank, params, top_n=TOP_N,
            stage1=lambda x, off, w: _stage1(x, off, w, params),
            stage2=lambda gc, gs: _stage2(gc, gs, params, u, port),
            full_rows=lambda full, rows: _full_rows(full, rows, params, u, port))
        assert ((params["top_k"] == 0) | (params["top_k"] > TOP_N)).sum() >= 2  # round 2 is exercised
        otok, ost = port.sample_batch(logits, params, None, None, None, u)
        assert np.array_equal(st.numpy(), ost), (st, ost)
        assert np.array_equal(tok.numpy(), otok), (rank, tok, otok)
        got = [torch.zeros_like(tok) for _ in range(2)]
        dist.all_gather(got, tok)
        assert torch.equal(got[0], got[1])  # every rank drew the same tokens
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_sharded_step_on_two_gloo_ranks():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port_no = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    try:
        mp.start_processes(_worker, args=(port_no, errq), nprocs=2, join=True, start_method="spawn")
    except Exception as e:
        msgs = []
        while not errq.empty():
            msgs.append(errq.get())
        pytest.fail(f"{e}\n" + "\n".join(msgs))


def test_shard_layout_partitions_the_vocabulary():
    from sixi_smp.sharded import ShardLayout

    for vocab in (1, 7, 3001, 151936):
        for n in (1, 2, 3, 8, 16):
            lay = ShardLayout(vocab, n)
            edges = [(lay.offset(r), lay.width(r)) for r in range(n)]
            assert edges[0][0] == 0 and sum(w for _, w in edges) == vocab
            assert all(edges[r][0] + edges[r][1] == edges[r + 1][0] for r in range(n - 1))
