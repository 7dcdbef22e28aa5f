"""Vocab-sharded sampling over torch.distributed: each rank holds a contiguous slice of the
vocabulary of every row (logits produced vocab-parallel). One step is

  stage 1   sixi_smp_shard_candidates on this rank's slice -> per-row best top_n and stats
  exchange  all-gather of both arrays (NCCL over NVLink on GPUs; rank-major layout)
  stage 2   sixi_smp_merge_shards, identical on every rank -> the token of every row

so every rank ends with the same tokens, as sixi_smp_sample on the full rows would draw them (exact
for top_k <= top_n; see the header for the rows that report SIXI_OUT_OF_BOUNDS).
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


def sample_vocab_sharded(shard_logits, layout: ShardLayout, rank: int, params, *, top_n: int = 64,
                         masks=None, hist=None, hist_off=None, uniforms=None, step: int = 0,
                         stage1: Callable | None = None, stage2: Callable | None = None, group=None,
                         sampler=None, stream=None):
    """One sharded sampling step on this rank. `shard_logits` are this rank's columns
    [n_rows, width(rank)] (a view into wider rows is fine). Returns (tokens, statuses)."""
    import torch
    import torch.distributed as dist

    if stage1 is None:
        def stage1(x, off, width):
            return sampler.shard_candidates(x, off, width, params, top_n=top_n, masks=masks, hist=hist,
                                            hist_off=hist_off, stream=stream)
    if stage2 is None:
        def stage2(gc, gs):
            return sampler.merge_shards(gc, gs, params, uniforms=uniforms, step=step, stream=stream)

    cand, stats = stage1(shard_logits, layout.offset(rank), layout.width(rank))
    world = layout.n_shards
    # gathered along dim 0 (rank-major), then viewed as [world, n_rows, ...]
    g_cand = torch.empty((world * cand.shape[0],) + tuple(cand.shape[1:]), dtype=cand.dtype, device=cand.device)
    g_stats = torch.empty((world * stats.shape[0],) + tuple(stats.shape[1:]), dtype=stats.dtype,
                          device=stats.device)
    dist.all_gather_into_tensor(g_cand, cand.contiguous(), group=group)
    dist.all_gather_into_tensor(g_stats, stats.contiguous(), group=group)
    return stage2(g_cand.view((world,) + tuple(cand.shape)), g_stats.view((world,) + tuple(stats.shape)))
