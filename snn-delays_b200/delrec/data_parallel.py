"""Batch-parallel training across GPUs (one process per GPU, torch.distributed).

The delay-LIF scan never splits time; samples are independent, so ranks hold the same
parameters and disjoint batch shards, and one all-reduce of a single flat fp32 bucket
of every parameter gradient per step keeps them identical (NCCL over NVLink on B200s;
gloo on CPU for the tests).  The reference trains one process per GPU without any
collective, so this has no counterpart there."""

from __future__ import annotations

import torch
import torch.distributed as dist


def allreduce_gradients(params, group=None, average=True):
    """Sum (then average) the gradients of ``params`` over the process group with one
    collective on a flat bucket; parameters without a gradient are skipped identically
    on every rank (their ``grad`` must be None everywhere)."""
    if not dist.is_available() or not dist.is_initialized():
        return
    ws = dist.get_world_size(group)
    if ws == 1:
        return
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    if average:
        flat.div_(ws)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def shard_batch(x, labels, rank, world_size, dim=1):
    """The rank's contiguous share of a (T, B, ...) batch along the batch dimension."""
    B = x.shape[dim]
    per = (B + world_size - 1) // world_size
    lo, hi = rank * per, min(B, (rank + 1) * per)
    return x.narrow(dim, lo, hi - lo), labels[lo:hi]
