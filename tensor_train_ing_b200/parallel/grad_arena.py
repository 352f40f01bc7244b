"""One flat fp32 gradient buffer for every fused weight group of a model.

The fused ops accumulate weight gradients into their group's buffer (``WeightGroup.sink_grad``);
placing those buffers back to back in one arena, in backward order, lets data parallelism
reduce all matrix gradients with a few large in-place collectives (and bucket them as blocks
finish their backward) instead of copying scattered ``.grad`` tensors.
"""
from __future__ import annotations

import torch

from ..ops.block import model_weight_groups
from ..ops.weights import group_for


class GradArena:
    def __init__(self, model, device):
        self.model = model
        specs = model_weight_groups(model)
        self.groups = []
        total = 0
        seen = set()
        for owner, name, lins in specs:
            params = [l.weight for l in lins]
            if any(not p.requires_grad for p in params) or any(id(p) in seen for p in params):
                continue  # frozen, or a tied embedding already placed through the other group
            seen.update(id(p) for p in params)
            grp = group_for(owner, name, params)
            n = sum(grp.rows) * grp.d_in
            self.groups.append((grp, total, n))
            total += n
        self.numel = total
        self.flat = torch.zeros(total, device=device, dtype=torch.float32)
        for grp, off, n in self.groups:
            grp._grad = self.flat[off:off + n].view(sum(grp.rows), grp.d_in)
        ids = {id(p) for grp, _, _ in self.groups for p in grp.params}
        self.other = [p for p in model.parameters() if p.requires_grad and id(p) not in ids]

    def arena_params(self):
        return [p for grp, _, _ in self.groups for p in grp.params]

    def zero_(self):
        """Reset: attach every group's views (zeroed) so backward accumulates with beta = 1."""
        self.flat.zero_()
        for grp, _, _ in self.groups:
            for p, v in zip(grp.params, grp._views(grp._grad)):
                p.grad = v
        for p in self.other:
            p.grad = None
