"""Owner-computes sharded data parallelism (the framework's counterpart of the reference's FSDP2 layer,
tnlm/parallel.py:23-44).

Semantics kept from the reference: gradients are SUMMED over ranks (divide factor 1), every rank
back-propagates ``local_loss_sum / global_valid_targets``, the global gradient norm is clipped, and
Muon orthogonalises each FULL logical matrix (never a row shard; the reference verifies this in
tests/test_distributed_muon.py:21-31).

Layout, chosen for 180 GB per GPU and NVLink/NVSwitch all-to-all bandwidth instead of per-block
FSDP unshards:

* Trainable parameters are grouped into *units*: one unit per fused weight group (the matrices a
  single GEMM consumes, e.g. q1|k1|q2|k2|v of a layer) and one per remaining parameter.  Units are
  assigned whole to ranks by a deterministic longest-first balance, so each rank owns complete
  matrices.
* One flat gradient buffer and one flat parameter buffer (the parameters' dtype, fp32) hold the units rank by rank:
  rank r's units occupy ``[r*S, (r+1)*S)``.  Every parameter's storage and ``.grad`` are views of
  these buffers; the fused backward GEMMs accumulate straight into them across micro-batches.
* After the last micro-batch ONE reduce-scatter (in place, NCCL) leaves each rank the summed
  gradients of the units it owns; the optimizer (whose state exists only for owned parameters)
  updates them; ONE all-gather (in place) brings every rank the updated parameters.  Per step that
  is 1 reduce-scatter + 1 all-gather of the model, where FSDP2 issues 2 all-gathers and a
  reduce-scatter per block per micro-batch.

On CUDA with NCCL the two flat buffers live in symmetric memory (mapped into every rank's address
space over NVLink) and both collectives are this framework's own kernels: the reduce-scatter pulls
each peer's copy of the local region and sums it in rank order (deterministic) while emitting the
sum of squares for the clip, and the all-gather pulls each owner's updated region while writing the
bf16 operand caches of the GEMM weights in the same pass.  A bounded cross-GPU barrier through
symmetric signal pads orders them.  ``TTB_PEER_COLLECTIVES=0`` selects NCCL instead.

With the gloo backend (CPU tests) the reduce-scatter is an all-reduce and the all-gather a
broadcast per rank region; the arithmetic is the same sum.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops.block import model_weight_groups
from ..ops.weights import group_for

ALIGN = 64  # elements: every unit and every rank region starts on a 256-byte boundary


def _aligned(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def assign_units(sizes: list[int], world: int) -> list[int]:
    """Owner rank of each unit: longest first onto the least-loaded rank (ties: lowest rank, then
    original unit order), so the assignment depends only on the sizes and the world size."""
    load = [0] * world
    owner = [0] * len(sizes)
    for i in sorted(range(len(sizes)), key=lambda k: (-sizes[k], k)):
        r = min(range(world), key=lambda q: (load[q], q))
        owner[i] = r
        load[r] += _aligned(sizes[i])
    return owner


class ShardedDataParallel:
    def __init__(self, model, device, group=None, *, fused: bool = True):
        self.model = model
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        self.backend = dist.get_backend(group) if dist_on else None
        device = torch.device(device)
        units, seen = [], set()
        if fused:
            for owner, name, lins in model_weight_groups(model):
                params = [l.weight for l in lins]
                if any(not p.requires_grad for p in params) or any(id(p) in seen for p in params):
                    continue
                seen.update(id(p) for p in params)
                units.append(("group", group_for(owner, name, params), params))
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                units.append(("param", p, [p]))
        sizes = [sum(p.numel() for p in params) for _, _, params in units]
        dtypes = {p.dtype for _, _, params in units for p in params}
        if len(dtypes) > 1:
            raise ValueError(f"sharded data parallelism needs one parameter dtype, got {sorted(map(str, dtypes))}")
        dtype = dtypes.pop() if dtypes else torch.float32
        self.owner = assign_units(sizes, self.world)
        load = [0] * self.world
        for i, n in enumerate(sizes):
            load[self.owner[i]] += _aligned(n)
        self.shard = _aligned(max(load) if load else 0)
        self.peer = (self.world > 1 and self.backend == "nccl" and device.type == "cuda" and fused
                     and dtype == torch.float32 and os.environ.get("TTB_PEER_COLLECTIVES", "1") != "0")
        if self.peer:
            self._init_symmetric(device, dtype)
        else:
            self.grad_flat = torch.zeros(self.world * self.shard, device=device, dtype=dtype)
            self.param_flat = torch.zeros(self.world * self.shard, device=device, dtype=dtype)
        cursor = [r * self.shard for r in range(self.world)]
        self.units = []
        with torch.no_grad():
            for (kind, obj, params), n, r in zip(units, sizes, self.owner):
                off = cursor[r]
                cursor[r] += _aligned(n)
                pos = off
                for p in params:
                    view = self.param_flat[pos:pos + p.numel()].view_as(p)
                    view.copy_(p.detach())
                    p.data = view
                    pos += p.numel()
                if kind == "group":
                    obj._grad = self.grad_flat[off:off + n].view(sum(obj.rows), obj.d_in)
                self.units.append((kind, obj, params, off, n, r))
        self.layout = [{"kind": k, "params": [self._name(p) for p in ps], "offset": off, "numel": n, "owner": r}
                       for k, _, ps, off, n, r in self.units]
        self._sq = None
        if self.peer:
            self._build_gather_plan()

    # ------------------------------------------------------------------ symmetric memory
    def _init_symmetric(self, device, dtype):
        # plain peer mappings only: these kernels use ordinary loads and stores, never multimem
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem
        group = self.group if self.group is not None else dist.group.WORLD
        enable = getattr(symm_mem, "enable_symm_mem_for_group", None)
        if enable is not None:
            enable(group.group_name)
        n = self.world * self.shard
        self.grad_flat = symm_mem.empty(n, dtype=dtype, device=device)
        self.param_flat = symm_mem.empty(n, dtype=dtype, device=device)
        self.grad_flat.zero_()
        self.param_flat.zero_()
        hg = symm_mem.rendezvous(self.grad_flat, group)
        hp = symm_mem.rendezvous(self.param_flat, group)
        self._handles = (hg, hp)
        self._gptrs = [int(x) for x in hg.buffer_ptrs]
        self._pptrs = [int(x) for x in hp.buffer_ptrs]
        self._pads = [int(x) for x in hg.signal_pad_ptrs]
        self._epoch = 0

    def _build_gather_plan(self):
        """Copy segments of the fused all-gather: every unit from its owner's buffer into the local
        one (own units are not copied), plus the bf16 cache of every weight group."""
        from ..ops._ext import lib
        rows, max_n = [], 0
        local = self.param_flat.data_ptr()
        for kind, obj, params, off, n, r in self.units:
            n4 = (n + 3) // 4 * 4  # units are 64-element aligned, so the rounded tail stays in padding
            src = self._pptrs[r] + 4 * off
            dst32 = 0 if r == self.rank else local + 4 * off
            dst16 = 0
            if kind == "group":
                cache = obj.bf16()  # allocates the cache; the gather refreshes it every step
                assert cache.numel() == n
                dst16 = cache.data_ptr()
            if dst32 == 0 and dst16 == 0:
                continue
            rows.append((src, dst32, dst16, n4 if dst16 == 0 else n))
            max_n = max(max_n, n4)
        self._segs = torch.tensor(rows, dtype=torch.int64).to(self.param_flat.device) if rows else None
        self._seg_max = max_n
        self._lib = lib

    def _barrier(self):
        self._epoch += 1
        self._lib().peer_barrier(self._pads, self.rank, self._epoch)

    def _name(self, p):
        if not hasattr(self, "_names"):
            self._names = {id(q): n for n, q in self.model.named_parameters()}
        return self._names.get(id(p), "?")

    # ------------------------------------------------------------------ ownership
    def owned_params(self) -> list[torch.Tensor]:
        return [p for _, _, params, _, _, r in self.units if r == self.rank for p in params]

    def owned_ids(self) -> set[int]:
        return {id(p) for p in self.owned_params()}

    def region(self, flat: torch.Tensor) -> torch.Tensor:
        return flat[self.rank * self.shard:(self.rank + 1) * self.shard]

    # ------------------------------------------------------------------ step phases
    def zero_grad(self):
        """Zero the gradient buffer and attach every parameter's ``.grad`` view (backward accumulates)."""
        self.grad_flat.zero_()
        for kind, obj, params, off, n, _ in self.units:
            pos = off
            for p in params:
                p.grad = self.grad_flat[pos:pos + p.numel()].view_as(p)
                pos += p.numel()

    def reduce_gradients(self):
        """Sum gradients over ranks; afterwards this rank's region holds its owned units' sums."""
        if self.world == 1:
            return
        self._sq = None
        if self.peer:
            self._barrier()  # every rank's backward has finished writing its buffer
            partial = self._lib().rs_reduce_sq(self._gptrs, self.rank * self.shard, self.region(self.grad_flat))
            self._sq = partial.sum()
        elif self.backend == "nccl":
            dist.reduce_scatter_tensor(self.region(self.grad_flat), self.grad_flat, group=self.group)
        else:
            dist.all_reduce(self.grad_flat, group=self.group)

    def grad_norm_sq(self) -> torch.Tensor:
        """Global sum of squared (reduced) gradients: owned regions, summed over ranks."""
        if self._sq is not None:  # emitted by the fused reduce-scatter
            sq = self._sq.clone()
        else:
            # one fused reduction in the gradients' dtype (as torch's clip_grad_norm_); no upcast copy
            sq = torch.linalg.vector_norm(self.region(self.grad_flat)).double().square()
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        return sq

    def clip_(self, max_norm: float) -> torch.Tensor:
        """Scale the owned gradients so the global norm is at most ``max_norm`` (the rule of
        torch.nn.utils.clip_grad_norm_); returns the pre-clip global norm (fp32, on the device)."""
        norm = self.grad_norm_sq().sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0).to(self.grad_flat.dtype)
        self.region(self.grad_flat).mul_(coef)
        return norm.float()

    def gather_params(self):
        """Bring every rank the owners' updated parameters."""
        if self.world == 1:
            return
        if self.peer:
            self._barrier()  # every owner has updated its region
            if self._segs is not None:
                self._lib().ag_pull_cast(self._segs, self._seg_max)
            for kind, obj, *_ in self.units:
                if kind == "group":
                    obj._key = obj._version_key()  # the caches were written from the gathered values
        elif self.backend == "nccl":
            dist.all_gather_into_tensor(self.param_flat, self.region(self.param_flat), group=self.group)
        else:
            ranks = dist.get_process_group_ranks(self.group) if self.group is not None else range(self.world)
            for r, global_rank in enumerate(ranks):
                dist.broadcast(self.param_flat[r * self.shard:(r + 1) * self.shard], src=global_rank,
                               group=self.group)
