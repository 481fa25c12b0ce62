"""Batch-parallel beam search across GPUs (one process per GPU).

Queries are independent, so the batch shards into contiguous query ranges:
every rank holds the full trie and head rows, generates (or receives) the
hidden states of its own queries -- global row ``q`` at level 0 and rows
``q*k .. q*k+k-1`` after -- runs the search locally, and the per-rank results
are concatenated with one all-gather per result tensor (NCCL over NVLink on
GPUs; gloo works the same way on CPU tensors).  There is no other exchange.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_queries(batch: int, rank: int, world: int) -> tuple[int, int]:
    """``(first_query, n_queries)`` of ``rank``'s contiguous shard."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    if batch % world:
        raise ValueError(f"batch {batch} does not divide evenly across {world} ranks")
    per = batch // world
    return rank * per, per


def level_rows(first_query: int, n_queries: int, level: int, beams: int) -> tuple[int, int]:
    """Global ``(first_row, rows)`` of a shard's hidden states at ``level``."""
    per_q = 1 if level == 0 else beams
    return first_query * per_q, n_queries * per_q


def gather_results(ids: torch.Tensor, logp: torch.Tensor, node: torch.Tensor, group=None,
                   out=None):
    """All-gather each rank's ``(ids (b*k, L), logp (b*k,), node (b*k,))`` into the
    full-batch tensors in rank order (pre-allocated ``out`` may be passed)."""
    world = dist.get_world_size(group)
    if out is None:
        out = (ids.new_empty((ids.shape[0] * world,) + tuple(ids.shape[1:])),
               logp.new_empty((logp.shape[0] * world,)),
               node.new_empty((node.shape[0] * world,)))
    for dst, src in zip(out, (ids, logp, node)):
        dist.all_gather_into_tensor(dst, src.contiguous(), group=group)
    return out
