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


class OverlappedAllReduce:
    """Gradient averaging that overlaps the backward: the parameters are split into
    buckets of about ``bucket_bytes`` (in reverse registration order, roughly the order
    autograd produces their gradients); when every gradient of a bucket has been
    accumulated, a post-accumulate-grad hook launches an asynchronous all-reduce of the
    bucket (with NCCL it runs on the collective stream while the backward of the earlier
    layers continues).  ``finish()`` waits for all of them, reduces any bucket whose
    gradients did not all arrive (the same way on every rank: buckets are reduced in a
    fixed order) and writes the averaged values back.  Call ``finish()`` after
    ``backward()`` and before the optimizer step, every step."""

    def __init__(self, params, group=None, bucket_bytes=2 << 20, average=True):
        self.group = group
        self.average = average
        self.params = [p for p in params if p.requires_grad]
        self.buckets = []
        cur, size = [], 0
        for p in reversed(self.params):
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self._bucket_of = {}
        for bi, b in enumerate(self.buckets):
            for p in b:
                self._bucket_of[id(p)] = bi
        self._ready = [0] * len(self.buckets)
        self._pending = {}
        self._hooks = []
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))

    def _launch(self, bi):
        grads = [p.grad for p in self.buckets[bi]]
        flat = torch.cat([g.reshape(-1) for g in grads])
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self._pending[bi] = (work, flat)

    def _on_grad(self, p):
        bi = self._bucket_of[id(p)]
        self._ready[bi] += 1
        if self._ready[bi] == len(self.buckets[bi]) and bi not in self._pending:
            self._launch(bi)

    def finish(self):
        if not self._hooks:
            return
        ws = dist.get_world_size(self.group)
        for bi in range(len(self.buckets)):
            if bi not in self._pending:
                if any(p.grad is None for p in self.buckets[bi]):
                    for p in self.buckets[bi]:
                        if p.grad is None:
                            p.grad = torch.zeros_like(p)
                self._launch(bi)
        for bi in range(len(self.buckets)):
            work, flat = self._pending[bi]
            work.wait()
            if self.average:
                flat.div_(ws)
            off = 0
            for p in self.buckets[bi]:
                n = p.grad.numel()
                p.grad.copy_(flat[off:off + n].view_as(p.grad))
                off += n
        self._pending.clear()
        self._ready = [0] * len(self.buckets)

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
