"""Data-parallel exchange for DCNv2 layers: batch-sharded training needs one
collective per step, a sum (or mean) all-reduce of every layer's weight and bias
gradients.  All gradients go into one flat fp32 bucket so the step issues a
single all-reduce (NCCL on GPUs, gloo on CPU); the bucket is reused across steps.

Usage (one process per GPU, ``torch.distributed`` initialised)::

    reducer = GradBucket([layer1, layer2, layer3])   # modules or parameters
    loss.backward()
    reducer.allreduce(average=True)                  # before optimizer.step()
"""
from __future__ import annotations

from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


def _params(objs: Iterable) -> List[torch.nn.Parameter]:
    out: List[torch.nn.Parameter] = []
    for o in objs:
        if isinstance(o, torch.nn.Module):
            out.extend(p for p in o.parameters() if p.requires_grad)
        else:
            out.append(o)
    return out


class GradBucket:
    """One flat fp32 bucket holding the gradients of `objs` (modules or tensors)."""

    def __init__(self, objs: Iterable, group: Optional[dist.ProcessGroup] = None):
        self.params = _params(objs)
        if not self.params:
            raise ValueError("GradBucket needs at least one parameter")
        self.group = group
        self.numel = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.buf = torch.zeros(self.numel, dtype=torch.float32, device=dev)

    def allreduce(self, average: bool = False) -> torch.Tensor:
        """Sums (or averages) the gradients over the process group in place."""
        off = 0
        for p in self.params:
            n = p.numel()
            if p.grad is None:
                self.buf[off:off + n].zero_()
            else:
                self.buf[off:off + n].copy_(p.grad.reshape(-1))
            off += n
        dist.all_reduce(self.buf, group=self.group)
        if average:
            self.buf.div_(dist.get_world_size(self.group))
        off = 0
        for p in self.params:
            n = p.numel()
            view = self.buf[off:off + n].view_as(p)
            if p.grad is None:
                p.grad = view.to(p.dtype).clone()
            else:
                p.grad.copy_(view)
            off += n
        return self.buf


def allreduce_tensors(tensors: List[torch.Tensor], group: Optional[dist.ProcessGroup] = None,
                      average: bool = False) -> List[torch.Tensor]:
    """Flat sum (mean) all-reduce of a list of tensors; returns fp32 copies of the results."""
    flat = torch.cat([t.reshape(-1).float() for t in tensors])
    dist.all_reduce(flat, group=group)
    if average:
        flat.div_(dist.get_world_size(group))
    out, off = [], 0
    for t in tensors:
        out.append(flat[off:off + t.numel()].view(t.shape))
        off += t.numel()
    return out
