"""Data-parallel exchange for DCNv2 layers.

Batch-sharded training of DCNv2 layers needs one collective per step: a sum (or
mean) all-reduce of every layer's weight and bias gradients.  Each sample's
forward, grad_input, grad_offset and grad_mask are independent of the other
ranks' samples, so nothing else crosses the ranks.

``GradBucket`` keeps one flat fp32 buffer with a slice (a "bucket") per module
or parameter it was given.  With ``overlap=True`` a bucket's all-reduce is
started, asynchronously, as soon as the last of its parameters has received its
gradient during ``backward()``: the layers run backward from the last to the
first, so the exchange of layer i overlaps the backward of layers i-1 ... 0
(NCCL runs the collective on its own stream, ordered after the gradient's
producer).  ``allreduce()`` then only waits for the outstanding collectives
(issuing any bucket whose hooks did not fire) and writes the reduced values back
into ``p.grad``.  Gradients are gathered into and scattered out of the buffer
with one multi-tensor copy per bucket, not one copy per parameter.

Usage (one process per GPU, ``torch.distributed`` initialised)::

    reducer = GradBucket([layer1, layer2, layer3], overlap=True, average=True)
    loss.backward()                                  # buckets start as grads arrive
    reducer.allreduce()                              # before optimizer.step()
"""
from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


def _param_groups(objs: Iterable) -> List[List[torch.nn.Parameter]]:
    groups: List[List[torch.nn.Parameter]] = []
    for o in objs:
        if isinstance(o, torch.nn.Module):
            ps = [p for p in o.parameters() if p.requires_grad]
        else:
            ps = [o]
        if ps:
            groups.append(ps)
    return groups


class GradBucket:
    """Flat fp32 buckets (one per module / parameter of `objs`) for the gradient
    all-reduce of data-parallel training, optionally overlapped with backward."""

    def __init__(self, objs: Iterable, group: Optional[dist.ProcessGroup] = None,
                 overlap: bool = False, average: bool = False):
        self.groups = _param_groups(objs)
        if not self.groups:
            raise ValueError("GradBucket needs at least one parameter")
        self.params = [p for g in self.groups for p in g]
        self.group = group
        self.average = average
        self.numel = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.buf = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        self.views: List[List[torch.Tensor]] = []
        off = 0
        for g in self.groups:
            vs = []
            for p in g:
                vs.append(self.buf[off:off + p.numel()].view(p.shape))
                off += p.numel()
            self.views.append(vs)
        self._bounds = []
        off = 0
        for g in self.groups:
            n = sum(p.numel() for p in g)
            self._bounds.append((off, off + n))
            off += n
        self._works: List[Optional[object]] = [None] * len(self.groups)
        self._pending = [0] * len(self.groups)
        self._handles = []
        if overlap:
            self._attach()

    # -- helpers
    def _avg_op(self):
        backend = dist.get_backend(self.group)
        return dist.ReduceOp.AVG if backend == "nccl" else None

    def _launch(self, i: int, average: bool) -> None:
        ps, vs = self.groups[i], self.views[i]
        have = [(v, p.grad) for v, p in zip(vs, ps) if p.grad is not None]
        missing = [v for v, p in zip(vs, ps) if p.grad is None]
        if have:
            torch._foreach_copy_([v for v, _ in have], [g for _, g in have])
        for v in missing:
            v.zero_()
        lo, hi = self._bounds[i]
        op = self._avg_op() if average else dist.ReduceOp.SUM
        self._works[i] = (dist.all_reduce(self.buf[lo:hi], op=op or dist.ReduceOp.SUM, group=self.group,
                                          async_op=True), average and op is None)

    def _attach(self) -> None:
        """Registers the hooks that start a bucket once all of its parameters have
        accumulated their gradient for this step."""
        for i, g in enumerate(self.groups):
            for p in g:
                def hook(_p, i=i):
                    self._pending[i] += 1
                    if self._pending[i] == len(self.groups[i]) and self._works[i] is None:
                        self._launch(i, self.average)
                self._handles.append(p.register_post_accumulate_grad_hook(hook))

    def detach(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles = []

    # -- public
    def allreduce(self, average: Optional[bool] = None) -> torch.Tensor:
        """Sums (or averages) the gradients over the process group in place.
        `average` defaults to the constructor's; buckets already started by the
        backward hooks (overlap) use the constructor's setting."""
        if average is None:
            average = self.average
        elif self._handles and average != self.average:
            raise ValueError("with overlap, choose sum or mean in the constructor (average=...)")
        world = dist.get_world_size(self.group)
        for i in range(len(self.groups)):
            if self._works[i] is None:
                self._launch(i, average)
        for i in range(len(self.groups)):
            work, divide = self._works[i]
            work.wait()
            if divide:
                lo, hi = self._bounds[i]
                self.buf[lo:hi].div_(world)
            ps, vs = self.groups[i], self.views[i]
            for p, v in zip(ps, vs):
                if p.grad is None:
                    p.grad = v.to(p.dtype).clone()
            torch._foreach_copy_([p.grad for p in ps], vs)
            self._works[i] = None
            self._pending[i] = 0
        return self.buf


def allreduce_tensors(tensors: List[torch.Tensor], group: Optional[dist.ProcessGroup] = None,
                      average: bool = False) -> List[torch.Tensor]:
    """Flat sum (mean) all-reduce of a list of tensors in one collective; returns
    fp32 views of the reduced values (one multi-tensor copy in, no concatenation)."""
    n = sum(t.numel() for t in tensors)
    flat = torch.empty(n, dtype=torch.float32, device=tensors[0].device)
    views, off = [], 0
    for t in tensors:
        views.append(flat[off:off + t.numel()].view(t.shape))
        off += t.numel()
    torch._foreach_copy_(views, list(tensors))
    if average and dist.get_backend(group) == "nccl":
        dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=group)
    else:
        dist.all_reduce(flat, group=group)
        if average:
            flat.div_(dist.get_world_size(group))
    return views
