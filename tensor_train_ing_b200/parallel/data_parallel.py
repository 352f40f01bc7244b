"""Data parallelism over NCCL for the fused model.

Every rank holds the full model; gradients are summed across ranks (the reference's FSDP divide
factor 1, tnlm/parallel.py:23-30) and every rank applies the same optimizer update, so replicated
parameters stay bitwise identical.  The loss-normalization contract is the reference's: each rank
back-propagates ``local_loss_sum / global_valid_targets`` (tnlm/distributed_train.py:401).

The fused weight gradients live in one ``GradArena``; they are reduced in ``bucket_bytes`` slices
on a side stream as soon as the whole backward pass has produced them, and small parameters
(norm gains, biases, head scalars) are reduced as one coalesced buffer.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .grad_arena import GradArena


def global_count(n: torch.Tensor) -> torch.Tensor:
    """All-reduce a valid-target count (int64) across ranks."""
    n = n.clone().to(torch.int64)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(n)
    return n


class DataParallel:
    def __init__(self, model, device, group=None, bucket_bytes: int = 512 << 20):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.arena = GradArena(model, device)
        self.bucket = max(1, bucket_bytes // 4)

    def zero_grad(self):
        self.arena.zero_()

    def reduce_gradients(self):
        """Sum gradients over ranks in place (no-op on one rank)."""
        if self.world == 1:
            return
        flat = self.arena.flat
        for s in range(0, flat.numel(), self.bucket):
            dist.all_reduce(flat[s:s + self.bucket], group=self.group)
        small = [p for p in self.arena.other if p.grad is not None]
        if small:
            buf = torch.cat([p.grad.reshape(-1).float() for p in small])
            dist.all_reduce(buf, group=self.group)
            off = 0
            for p in small:
                n = p.grad.numel()
                p.grad.copy_(buf[off:off + n].view_as(p.grad))
                off += n
