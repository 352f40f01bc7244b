"""Weight groups: bf16 operand caches and fused fp32 gradient accumulation for the sm_100a ops.

Parameters stay fp32 masters (as under the reference's bf16 autocast).  A ``WeightGroup`` is a
list of parameters that one GEMM consumes together (e.g. q1, k1, q2, k2, v of a layer):

* ``bf16()`` returns the row-concatenated bf16 copy, rebuilt only when a parameter changed
  (tracked through the tensors' version counters), i.e. once per optimizer step rather than
  once per micro-batch as autocast would;
* ``sink_grad(compute)`` runs the weight-gradient GEMM straight into one fp32 buffer
  ([rows, d_in]) whose row blocks are attached as the parameters' ``.grad`` views: the first
  micro-batch of a step overwrites (beta = 0), later ones accumulate in the GEMM epilogue
  (beta = 1), so no separate gradient-accumulation kernel runs.  If the parameters' grads are
  not this group's views (set by someone else), the gradient is returned to autograd instead.

Under parameter-sharded data parallelism the group is attached to its sharding layer
(``_shard``): the gradient then goes to the layer's per-layer staging buffer and the layer reduces
it onto the owning rank.
"""
from __future__ import annotations

import torch
from torch.optim.optimizer import register_optimizer_step_post_hook

# Optimizer steps seen so far (every torch optimizer, through a global step post-hook).  Part of the
# cache key: fused optimizer kernels (torch's fused AdamW among them) update parameters in place
# without bumping their version counters, so a version-only key would keep serving the bf16 copy
# of the weights from before the step.
_STEPS = [0]


def weights_updated():
    """Invalidate every bf16 weight cache (called after each optimizer step; call it after any other
    in-place parameter update that bypasses autograd's version counters)."""
    _STEPS[0] += 1


register_optimizer_step_post_hook(lambda optimizer, args, kwargs: weights_updated())


class WeightGroup:
    def __init__(self, params: list[torch.Tensor]):
        self.params = list(params)
        d_in = {p.shape[-1] for p in self.params}
        if len(d_in) != 1:
            raise ValueError("a weight group needs a common input dimension")
        self.rows = [p.shape[0] for p in self.params]
        self.d_in = d_in.pop()
        self._cache = None
        self._key = None
        self._grad = None
        self._shard = None  # (sharding layer, unit) under parameter-sharded data parallelism
        self._gather = None  # parallel.gather.GatheredWeight when the bf16 rows are sharded across ranks

    # ------------------------------------------------------------------ forward operand
    def _version_key(self):
        return (_STEPS[0],) + tuple((p.data_ptr(), p._version) for p in self.params)

    def operand(self):
        """(bf16 weight, gather description or None) for a GEMM that can gather row-sharded weights
        itself: with a description, the returned staging buffer is filled by that GEMM."""
        if self._gather is not None:
            return self._gather.operand()
        return self.bf16(), None

    def bf16(self) -> torch.Tensor:
        if self._gather is not None:
            return self._gather.resident()
        if self._shard is not None and self._cache is not None:
            return self._cache  # written by the sharding layer's gather, once per optimizer step
        key = self._version_key()
        if self._cache is None or key != self._key:
            with torch.no_grad():
                if self._cache is None or self._cache.device != self.params[0].device:
                    self._cache = torch.empty(sum(self.rows), self.d_in, device=self.params[0].device,
                                              dtype=torch.bfloat16)
                row = 0
                for p, n in zip(self.params, self.rows):
                    self._cache[row:row + n].copy_(p.detach())
                    row += n
            self._key = key
        return self._cache

    # ------------------------------------------------------------------ backward sink
    def _grad_buffer(self):
        dev = self.params[0].device
        if self._grad is None or self._grad.device != dev:
            self._grad = torch.empty(sum(self.rows), self.d_in, device=dev, dtype=torch.float32)
        return self._grad

    def _views(self, buf):
        return list(buf.split(self.rows, dim=0))

    def sink_grad(self, compute):
        """compute(out_fp32 [rows, d_in], beta) writes (beta=0) or adds (beta=1) the weight grad.

        Returns the list of gradients to hand to autograd (None where accumulated in place)."""
        if self._shard is not None:
            layer, unit = self._shard
            return layer.sink(unit, compute)
        leafs = all(p.is_leaf and p.requires_grad for p in self.params)
        if leafs:
            buf = self._grad_buffer()
            views = self._views(buf)
            if all(p.grad is None for p in self.params):
                compute(buf, 0.0)
                for p, v in zip(self.params, views):
                    p.grad = v
                return [None] * len(self.params)
            if all(p.grad is not None and p.grad.data_ptr() == v.data_ptr() and p.grad.shape == v.shape
                   for p, v in zip(self.params, views)):
                compute(buf, 1.0)
                return [None] * len(self.params)
        out = torch.empty(sum(self.rows), self.d_in, device=self.params[0].device, dtype=torch.float32)
        compute(out, 0.0)
        return [g.to(p.dtype) for g, p in zip(self._views(out), self.params)]


class SpectralWeights:
    """The weight group of SpectralLinear layers on the fused path.

    ``bf16()`` writes bf16(gamma W / sigma) of every layer with one kernel pass each (sigma = u^T W v
    reduced on the device), cached until a weight, gamma, u or v changes or an optimizer steps;
    ``sink_grad`` turns the weight-gradient GEMM's dW_eff into dW and dgamma with the spectral
    backward kernel (the gradient through sigma included).  ``params`` lists each layer's weight and
    gamma, in that order."""

    def __init__(self, linears):
        self.linears = list(linears)
        self.params = [t for lin in self.linears for t in (lin.weight, lin.gamma)]
        self.rows = [lin.weight.shape[0] for lin in self.linears]
        self.d_in = self.linears[0].weight.shape[1]
        self._cache = None
        self._key = None
        self._sigmas: list[torch.Tensor] = []

    def _version_key(self):
        return (_STEPS[0],) + tuple((t.data_ptr(), t._version) for lin in self.linears
                                    for t in (lin.weight, lin.gamma, lin.u, lin.v))

    def operand(self):
        return self.bf16(), None

    def bf16(self) -> torch.Tensor:
        from ..models.normalization import SIGMA_FLOOR
        from ._ext import lib
        key = self._version_key()
        if self._cache is None or key != self._key:
            dev = self.linears[0].weight.device
            if self._cache is None or self._cache.device != dev:
                self._cache = torch.empty(sum(self.rows), self.d_in, device=dev, dtype=torch.bfloat16)
            self._sigmas, row = [], 0
            with torch.no_grad():
                for lin, n in zip(self.linears, self.rows):
                    self._sigmas.append(lib().spectral_cast(lin.weight.detach(), lin.gamma.detach(), lin.u, lin.v,
                                                            SIGMA_FLOOR, self._cache[row:row + n]))
                    row += n
            self._key = key
        return self._cache

    def sink_grad(self, compute):
        from ..models.normalization import SIGMA_FLOOR
        from ._ext import lib
        eff = torch.empty(sum(self.rows), self.d_in, device=self.linears[0].weight.device, dtype=torch.float32)
        compute(eff, 0.0)
        self.bf16()  # the sigmas of the weights this backward differentiates
        grads, row = [], 0
        for lin, n, sigma in zip(self.linears, self.rows, self._sigmas):
            dw, dgamma = lib().spectral_grad(eff[row:row + n], lin.weight.detach(), lin.gamma.detach(), lin.u,
                                             lin.v, sigma, SIGMA_FLOOR)
            grads += [dw, dgamma]
            row += n
        return grads


def spectral_group_for(owner, name: str, linears):
    """Cached SpectralWeights stored on ``owner`` (rebuilt if the layer objects changed)."""
    attr = f"_ttb_spectral_{name}"
    grp = getattr(owner, attr, None)
    if grp is None or len(grp.linears) != len(linears) or any(a is not b for a, b in zip(grp.linears, linears)):
        grp = SpectralWeights(linears)
        object.__setattr__(owner, attr, grp)
    return grp


def group_for(owner, name: str, params: list[torch.Tensor]):
    """Cached WeightGroup stored on ``owner`` (rebuilt if the parameter objects changed)."""
    attr = f"_ttb_group_{name}"
    grp = getattr(owner, attr, None)
    if grp is None or len(grp.params) != len(params) or any(a is not b for a, b in zip(grp.params, params)):
        grp = WeightGroup(params)
        object.__setattr__(owner, attr, grp)
    return grp


def cache_views(model):
    """Rows of the bf16 operand caches an optimizer can write the updated weights into.

    Returns ({id(param): bf16 [rows, d_in] view into its group's cache}, [groups]) over the weight
    groups whose cache already exists and is managed here (not by a parameter-sharding layer)."""
    from .block import model_weight_groups
    views, groups = {}, []
    for owner, name, lins in model_weight_groups(model):
        grp = getattr(owner, f"_ttb_group_{name}", None)
        if (grp is None or grp._cache is None or grp._shard is not None
                or any(p is not l.weight for p, l in zip(grp.params, lins))):
            continue
        row = 0
        for p, n in zip(grp.params, grp.rows):
            views[id(p)] = grp._cache[row:row + n]
            row += n
        groups.append(grp)
    return views, groups


def mark_current(groups, written: set) -> None:
    """Declare the caches of groups whose every parameter's rows were just rewritten up to date."""
    for grp in groups:
        if all(id(p) in written for p in grp.params):
            grp._key = grp._version_key()
