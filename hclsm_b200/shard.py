"""Sequence sharding of the scan across the GPUs of one node.

Sequences (batch x slot) are independent, so a job of ``nseq`` sequences is cut
into contiguous per-rank shards and no collective sits on the data path.  The
one real exchange of a training step is the parameter gradient dA_log (and dD),
a (d_inner, d_state) fp32 sum over every sequence: one all-reduce of 128 KB at
d_inner=2048, d_state=16.  ``gather_shards`` (all-gather) exists for
verification only.  Works with any torch.distributed backend (NCCL on GPUs,
gloo for the host-side tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) of n items for rank; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    q, r = divmod(n, world)
    start = rank * q + min(rank, r)
    return start, start + q + (1 if rank < r else 0)


def allreduce_param_grads(grads, group=None):
    """Sum parameter gradients (e.g. dA_log, dD) over ranks in place."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return grads
    for g in grads:
        if g is not None:
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group)
    return grads


def gather_shards(t: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather per-rank shards along dim 0 into the full (n_total, ...) tensor."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return t
    sizes = [shard_range(n_total, r, world) for r in range(world)]
    m = max(e - s for s, e in sizes)
    pad = torch.zeros((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    return torch.cat([b[: e - s] for b, (s, e) in zip(bufs, sizes)], 0)


def sharded_scan_grads(compute, inputs: dict, n_total: int, group=None):
    """Run ``compute(shard_inputs) -> dict of grads`` on this rank's shard and
    combine: per-sequence gradients stay sharded, dA_log / dD are all-reduced."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    s, e = shard_range(n_total, rank, world)
    shard = {k: (v[s:e] if k not in ("A_log", "D") else v) for k, v in inputs.items()}
    out = compute(shard)
    allreduce_param_grads([out.get("dA_log"), out.get("dD")], group)
    return out, (s, e)
