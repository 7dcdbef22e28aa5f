"""Vocab-sharded sampling over torch.distributed: each rank holds a contiguous slice of the
vocabulary of every row (logits produced vocab-parallel). One step is

  stage 1   sixi_smp_shard_candidates on this rank's slice -> per-row best top_n and stats
  exchange  all-gather of both arrays (NCCL over NVLink on GPUs; rank-major layout)
  stage 2   sixi_smp_merge_shards, identical on every rank -> the token of every row
  round 2   only for rows whose kept set or draw reaches past the gathered candidates (stage 2
            reports SIXI_OUT_OF_BOUNDS, which can happen for top_k = 0 or top_k > top_n): their
            slices are packed (sixi_smp_gather_rows) and all-gathered, every rank rebuilds the full
            rows and samples them with sixi_smp_sample_indexed (each as its batch row)

so every rank ends with the same tokens, as sixi_smp_sample on the full rows draws them, for every
row. The flagged rows are the same on every rank (stage 2 is deterministic on identical data), so
every rank makes the same collective calls.
The stage functions are parameters so that the collective plumbing can be exercised on CPU
ranks (gloo) with host restatements of the two stages.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable


@dataclass(frozen=True)
class ShardLayout:
    """Rank r owns ids [offset(r), offset(r) + width(r)) of a vocabulary of `vocab` ids split
    over `n_shards` ranks (the first vocab % n_shards ranks hold one id more)."""

    vocab: int
    n_shards: int

    def width(self, r: int) -> int:
        base, extra = divmod(self.vocab, self.n_shards)
        return base + (1 if r < extra else 0)

    def offset(self, r: int) -> int:
        base, extra = divmod(self.vocab, self.n_shards)
        return r * base + min(r, extra)


OUT_OF_BOUNDS = 2


def sample_vocab_sharded(shard_logits, layout: ShardLayout, rank: int, params, *, top_n: int = 64,
                         masks=None, hist=None, hist_off=None, uniforms=None, step: int = 0,
                         stage1: Callable | None = None, stage2: Callable | None = None,
                         full_rows: Callable | None = None, group=None, sampler=None, stream=None,
                         mark: Callable | None = None):
    """One sharded sampling step on this rank. `shard_logits` are this rank's columns
    [n_rows, width(rank)] (a view into wider rows is fine). Returns (tokens, statuses).
    `full_rows(logits, rows)` samples rebuilt full rows `rows` (round 2); by default
    sixi_smp_sample on this rank's sampler with the rows' parameters, masks, histories and
    uniforms. `mark(name)`, when given, is called after stage 1, the exchange, stage 2 and round 2
    (a timer records a CUDA event there)."""
    import torch
    import torch.distributed as dist

    if full_rows is None:
        def full_rows(full, rows):
            # sixi_smp_sample_indexed: rebuilt row j is sampled as batch row rows[j], with the batch's
            # own parameter, mask, history and uniform arrays
            n = shard_logits.shape[0]
            t = torch.empty(n, dtype=torch.int32, device=full.device)
            st = torch.empty(n, dtype=torch.int32, device=full.device)
            sampler.sample_indexed(full, rows.to(torch.int32), params, t, st, masks=masks, hist=hist,
                                   hist_off=hist_off, uniforms=uniforms, step=step, stream=stream)
            return t[rows], st[rows]

    if stage1 is None:
        def stage1(x, off, width):
            return sampler.shard_candidates(x, off, width, params, top_n=top_n, masks=masks, hist=hist,
                                            hist_off=hist_off, stream=stream)
    if stage2 is None:
        def stage2(gc, gs):
            return sampler.merge_shards(gc, gs, params, uniforms=uniforms, step=step, stream=stream)

    if mark is None:
        def mark(name):
            return None
    cand, stats = stage1(shard_logits, layout.offset(rank), layout.width(rank))
    mark("stage1")
    world = layout.n_shards
    # gathered along dim 0 (rank-major), then viewed as [world, n_rows, ...]
    g_cand = torch.empty((world * cand.shape[0],) + tuple(cand.shape[1:]), dtype=cand.dtype, device=cand.device)
    g_stats = torch.empty((world * stats.shape[0],) + tuple(stats.shape[1:]), dtype=stats.dtype,
                          device=stats.device)
    dist.all_gather_into_tensor(g_cand, cand.contiguous(), group=group)
    dist.all_gather_into_tensor(g_stats, stats.contiguous(), group=group)
    mark("exchange")
    tok, sts = stage2(g_cand.view((world,) + tuple(cand.shape)), g_stats.view((world,) + tuple(stats.shape)))
    mark("stage2")
    # round 2: the rows stage 2 could not certify, sampled from their rebuilt full rows
    rows = (sts == OUT_OF_BOUNDS).nonzero().flatten()
    n_f = int(rows.numel())
    if n_f:
        wmax = max(layout.width(r) for r in range(world))
        part = torch.zeros((n_f, wmax), dtype=shard_logits.dtype, device=shard_logits.device)
        if sampler is not None:
            sampler.gather_rows(shard_logits, rows.to(torch.int32), layout.width(rank), out=part, stream=stream)
        else:
            part[:, :layout.width(rank)] = shard_logits[rows.to(shard_logits.device)]
        g_rows = torch.empty((world * n_f, wmax), dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(g_rows, part, group=group)
        g_rows = g_rows.view(world, n_f, wmax)
        full = torch.cat([g_rows[r, :, :layout.width(r)] for r in range(world)], dim=1).contiguous()
        t2, s2 = full_rows(full, rows)
        tok = tok.clone()
        sts = sts.clone()
        tok[rows] = t2.to(tok.device)
        sts[rows] = s2.to(sts.device)
    mark("round2")
    return tok, sts
