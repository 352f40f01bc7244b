"""Data parallelism (reference tnlm/parallel.py:23-44): the loss-normalization contract helpers and the
owner-computes sharded layer."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .sharded import ShardedDataParallel, assign_units  # noqa: F401


def global_count(n: torch.Tensor, group=None) -> torch.Tensor:
    """All-reduce a valid-target count (int64) across ranks: the denominator every rank divides its
    local loss sum by before backward (the loss-normalization contract)."""
    n = n.clone().to(torch.int64)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(n, group=group)
    return n


def full_state_dict(model) -> dict:
    """The complete model state on this rank's CPU (parameters are replicated between steps)."""
    return {k: v.detach().cpu().clone() for k, v in model.state_dict().items()}
