"""Vocab-sharded sampling across GPUs (NCCL all-gather between the two stages, and the second
exchange round for the rows the candidates cannot certify). Runs when the box has at least two
GPUs: one process per GPU, each holding 1/N of the vocabulary of every row. Every rank must draw
the same tokens, and they must be the oracle's for the full rows, every row."""

from __future__ import annotations

import datetime
import socket

import numpy as np
import pytest

from conftest import REPO, has_gpu

pytestmark = pytest.mark.gpu


def _ngpu() -> int:
    if not has_gpu():
        return 0
    import torch

    return torch.cuda.device_count()


def _worker(rank: int, world: int, port_no: int, errq):
    import os
    import sys

    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "sixi-asi_b200"))
    sys.path.insert(0, str(REPO / "tests"))
    import torch
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port_no)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        import sixi_smp as S
        from oracle import binding
        from sixi_smp import workloads as W
        from sixi_smp.sharded import ShardLayout, sample_vocab_sharded

        d = W.config2(rows=16, seed=900)
        vocab = d["logits"].shape[1]
        u = np.random.default_rng(3).random(16)
        lay = ShardLayout(vocab, world)
        full = torch.from_numpy(d["logits"]).to(dev)
        mine = full[:, lay.offset(rank):lay.offset(rank) + lay.width(rank)]
        params = torch.from_numpy(d["params"].view(np.uint8)).to(dev)
        hist = torch.from_numpy(d["hist"]).to(dev)
        hoff = torch.from_numpy(d["hist_off"]).to(dev)
        smp = S.Sampler(rank, 64, vocab)
        tok, st = sample_vocab_sharded(mine, lay, rank, params, top_n=64, hist=hist, hist_off=hoff,
                                       uniforms=torch.from_numpy(u).to(dev), sampler=smp)
        torch.cuda.synchronize()
        got = [torch.zeros_like(tok) for _ in range(world)]
        dist.all_gather(got, tok)
        assert all(torch.equal(got[0], g) for g in got), "ranks disagree"
        tok, st = tok.cpu().numpy(), st.cpu().numpy()
        port = binding.port()
        otok, ost = port.sample_batch(d["logits"], d["params"], None, d["hist"], d["hist_off"], u)
        assert (d["params"]["top_k"] == 0).sum() >= 2  # the second round is exercised
        for r in range(16):
            assert st[r] == ost[r] and tok[r] == otok[r], (r, tok[r], otok[r])
        smp.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.skipif(_ngpu() < 2, reason="needs at least two GPUs")
def test_vocab_sharded_over_nccl():
    import torch.multiprocessing as mp

    world = min(_ngpu(), 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port_no = s.getsockname()[1]
    errq = mp.get_context("spawn").SimpleQueue()
    try:
        mp.start_processes(_worker, args=(world, port_no, errq), nprocs=world, join=True, start_method="spawn")
    except Exception as e:
        msgs = []
        while not errq.empty():
            msgs.append(errq.get())
        pytest.fail(f"{e}\n" + "\n".join(msgs))
