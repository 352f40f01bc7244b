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

Parameter-sharded mode (``shard_params=True``; the counterpart of FSDP2 full sharding for models
whose fp32 parameters and gradients do not fit replicated, e.g. the 32B configuration): the GEMM
weight groups of the blocks and the unembedding become *sharded units*.  Their fp32 masters,
gradient accumulators and optimizer state exist only on the owning rank (buffers ``sp_param`` /
``sp_grad``); every rank keeps only what the kernels read, the bf16 operand caches, which the
per-step gather writes straight from the owners' masters.  Gradients leave each rank layer by layer:
the weight-gradient GEMMs of a block write into a per-block staging slot (two slots alternate), and
as soon as a block's last weight gradient is written the owners pull the block's slot from every
rank and add the rank-ordered sum into their accumulators (peer memory and a bounded barrier on
CUDA, an all-reduce elsewhere).  Per micro-batch each rank therefore moves its owned share of the
model gradient once over NVLink, and the model is materialised from the streamed serial
initialisation (models/init_stream.py) without any rank holding all fp32 weights.  Off the fused
path (CPU tests) the non-owned parameters are full fp32 compute copies refreshed by the gather, and
gradients reach the staging step through post-accumulate hooks.
"""
from __future__ import annotations

import os
import re

import torch
import torch.distributed as dist

from ..ops.block import model_weight_groups
from ..ops.weights import group_for

ALIGN = 64  # elements: every unit and every rank region starts on a 256-byte boundary
BARRIER_LIMIT_CYCLES = 20_000_000_000  # per-layer waits: about ten seconds of SM clock
PULL_BLOCKS = 64  # CTAs of a per-layer gradient pull: enough loads in flight for NVLink, most SMs left
                  # to the backward GEMMs running beside it


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


def _bucket_key(name: str) -> str:
    m = re.match(r"blocks\.(\d+)\.", name)
    return f"blocks.{m.group(1)}" if m else name.split(".")[0]


class _SUnit:
    """A sharded unit: one weight group whose master lives on one rank."""

    def __init__(self, index, group, params, names, owner, bucket):
        self.index, self.group, self.params, self.names = index, group, params, names
        self.owner, self.bucket = owner, bucket
        self.n = sum(p.numel() for p in params)
        self.stage_off = 0   # offset inside the bucket's staging slot
        self.goff = 0        # offset inside the owner's sp_param / sp_grad
        self.pending = len(params)


class _Bucket:
    """The sharded units of one block (or of the unembedding), staged and reduced together."""

    def __init__(self, index, key):
        self.index, self.key = index, key
        self.units: list[_SUnit] = []
        self.numel = 0
        self.own_off: list[int] = []   # per rank: first staging offset of the rank's units
        self.own_n: list[int] = []     # per rank: aligned size of the rank's units (contiguous)
        self.own_goff: list[int] = []  # per rank: matching offset in that rank's sp buffers
        self.cut: list[int] = []       # reduction slices (peer transport): rank r reduces [cut[r], cut[r+1])
        self.rd_off: list[int] = []    # per rank: offset of its slice of this bucket in that rank's rd_grad
        self.ready = 0


class ShardedDataParallel:
    def __init__(self, model, device, group=None, *, fused: bool = True, shard_params: bool = False,
                 init: str = "serial"):
        """``init`` (meta-device models): "serial" streams the CPU initialisation ``TensorLM(cfg)``
        would draw under the current seed; "device" draws the same distributions on the device."""
        self.model = model
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        self.backend = dist.get_backend(group) if dist_on else None
        self._ranks = (list(dist.get_process_group_ranks(group)) if dist_on and group is not None
                       else list(range(self.world)))
        device = torch.device(device)
        self.device = device
        self.fused = fused
        self.shard_params = bool(shard_params)
        self._names = {id(q): n for n, q in model.named_parameters()}
        meta = any(p.is_meta for p in model.parameters())
        if meta and not self.shard_params:
            raise ValueError("a meta-device model is materialised only by the parameter-sharded mode")

        units, sspec, seen = [], [], set()
        embed_id = id(model.embed.weight)  # read in fp32 by the embedding kernel: never sharded
        if fused or self.shard_params:
            for owner, name, lins in model_weight_groups(model):
                params = [l.weight for l in lins]
                if any(not p.requires_grad for p in params) or any(id(p) in seen for p in params):
                    continue
                if self.shard_params and all(id(p) != embed_id for p in params):
                    seen.update(id(p) for p in params)
                    sspec.append((group_for(owner, name, params), params))
                elif fused:
                    seen.update(id(p) for p in params)
                    units.append(("group", group_for(owner, name, params), params))
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                units.append(("param", p, [p]))
        sizes = [sum(p.numel() for p in params) for _, _, params in units]
        ssizes = [sum(p.numel() for p in params) for _, params in sspec]
        dtypes = {p.dtype for _, _, params in units for p in params} | {p.dtype for _, ps in sspec for p in ps}
        if len(dtypes) > 1:
            raise ValueError(f"sharded data parallelism needs one parameter dtype, got {sorted(map(str, dtypes))}")
        dtype = dtypes.pop() if dtypes else torch.float32
        self.dtype = dtype
        # one longest-first balance over every unit, so optimizer work and state are balanced
        owners = assign_units(sizes + ssizes, self.world)
        self.owner, s_owner = owners[:len(sizes)], owners[len(sizes):]
        load = [0] * self.world
        for i, n in enumerate(sizes):
            load[self.owner[i]] += _aligned(n)
        self.shard = max(_aligned(max(load) if load else 0), ALIGN)
        self.peer = (self.world > 1 and self.backend == "nccl" and device.type == "cuda" and fused
                     and dtype == torch.float32 and os.environ.get("TTB_PEER_COLLECTIVES", "1") != "0")
        # rank regions of the replicated flat buffers: equal (padded to the largest) for NCCL's
        # reduce-scatter / all-gather, packed back to back for the peer kernels
        if self.peer:
            self._rlen = [_aligned(x) for x in load]
            self._rstart = [sum(self._rlen[:r]) for r in range(self.world)]
            self._flat_len = max(sum(self._rlen), ALIGN)
        else:
            self._rlen = [self.shard] * self.world
            self._rstart = [r * self.shard for r in range(self.world)]
            self._flat_len = self.world * self.shard
        self._cache_mode = self.shard_params and fused  # non-owned weights exist only as bf16 caches
        self._build_sharded_layout(sspec, s_owner)
        # fused all-gather (parallel/gather.py): the bf16 rows of the sharded groups are split across the
        # ranks and gathered by the GEMMs that read them, instead of a full bf16 copy on every rank
        # (default on with the peer transport; a one-rank CUDA engine takes it with TTB_FUSED_GATHER=1, which
        # runs the whole path against its own memory)
        want = os.environ.get("TTB_FUSED_GATHER", "1" if self.peer else "0") != "0"
        self.fused_gather = (want and self._cache_mode and (self.peer or (self.world == 1 and device.type == "cuda"))
                             and all(sum(su.group.rows) % 64 == 0 and su.group.d_in % 8 == 0 for su in self.sunits))
        self.window = None
        if self.fused_gather and not self.peer:
            self._init_row_shards(device)
        if self.peer:
            self._init_symmetric(device, dtype)
        else:
            self.grad_flat = torch.zeros(self._flat_len, device=device, dtype=dtype)
            self.param_flat = torch.zeros(self._flat_len, device=device, dtype=dtype)
            self.sp_param = torch.zeros(self.s_shard, device=device, dtype=dtype)
            self.stage = (torch.zeros(2 * self.max_bucket, device=device, dtype=torch.float32)
                          if self._cache_mode else None)
        self.sp_grad = torch.zeros(self.s_shard, device=device, dtype=dtype)

        # ---------------------------------------------------------------- storage and values
        dest = {}  # parameter name -> tensor its initial value is copied into (None: placeholder)
        cursor = list(self._rstart)
        self.units = []
        for (kind, obj, params), n, r in zip(units, sizes, self.owner):
            off = cursor[r]
            cursor[r] += _aligned(n)
            pos = off
            for p in params:
                dest[self._names[id(p)]] = (p, self.param_flat[pos:pos + p.numel()].view(p.shape))
                pos += p.numel()
            if kind == "group":
                obj._grad = self.grad_flat[off:off + n].view(sum(obj.rows), obj.d_in)
            self.units.append((kind, obj, params, off, n, r))
        self._zero = torch.zeros((), device=device, dtype=dtype)
        for su in self.sunits:
            pos = su.goff
            for p, name in zip(su.params, su.names):
                if su.owner == self.rank:
                    dest[name] = (p, self.sp_param[pos:pos + p.numel()].view(p.shape))
                elif self._cache_mode:
                    dest[name] = (p, None)
                else:
                    dest[name] = (p, torch.empty(p.shape, device=device, dtype=dtype))
                pos += p.numel()
            su.group._shard = (self, su)
        if init not in ("serial", "device"):
            raise ValueError(f"unknown initialisation {init!r}")
        self._materialize(model, dest, meta, init)
        if self._cache_mode and any(su.owner != self.rank for su in self.sunits):
            model._ttb_weights_remote = True
        self.layout = ([{"kind": k, "params": [self._name(p) for p in ps], "offset": off, "numel": n, "owner": r}
                        for k, _, ps, off, n, r in self.units]
                       + [{"kind": "sharded", "params": su.names, "offset": su.goff, "numel": su.n,
                           "owner": su.owner, "bucket": self.buckets[su.bucket].key} for su in self.sunits])
        self._sq = None
        self._hooks = []
        if self.shard_params and not self._cache_mode:
            for su in self.sunits:
                for p in su.params:
                    self._hooks.append(p.register_post_accumulate_grad_hook(
                        lambda p, su=su: self._param_ready(su, p)))
        if self.peer:
            self._build_gather_plan()
        if self.shard_params:
            self.gather_params()  # caches / compute copies from the owners' initial masters

    # ------------------------------------------------------------------ layout
    def _build_sharded_layout(self, sspec, s_owner):
        self.sunits, self.buckets = [], []
        keys = {}
        for i, ((grp, params), r) in enumerate(zip(sspec, s_owner)):
            names = [self._names[id(p)] for p in params]
            key = _bucket_key(names[0])
            if key not in keys:
                keys[key] = len(self.buckets)
                self.buckets.append(_Bucket(len(self.buckets), key))
            su = _SUnit(i, grp, params, names, r, keys[key])
            self.sunits.append(su)
            self.buckets[su.bucket].units.append(su)
        gcur = [0] * self.world
        self.max_bucket = 0
        for b in self.buckets:
            b.units.sort(key=lambda u: (u.owner, u.index))
            off = 0
            b.own_off, b.own_n, b.own_goff = [0] * self.world, [0] * self.world, [0] * self.world
            for r in range(self.world):
                b.own_off[r], b.own_goff[r] = off, gcur[r]
                for su in b.units:
                    if su.owner == r:
                        su.stage_off, su.goff = off, gcur[r]
                        off += _aligned(su.n)
                        gcur[r] += _aligned(su.n)
                b.own_n[r] = off - b.own_off[r]
            b.numel = off
            self.max_bucket = max(self.max_bucket, off)
        self.s_shard = max(_aligned(max(gcur) if gcur else 0), ALIGN)
        self.max_bucket = max(self.max_bucket, ALIGN)
        # Peer transport: every rank reduces an equal slice of every bucket (whole-matrix ownership
        # would leave one rank pulling two 151M-parameter matrices of a block while the others idle),
        # into its rd_grad; owners gather their units' pieces from the slice holders once per step.
        for b in self.buckets:
            b.cut = [min(b.numel, (b.numel * r // self.world) // ALIGN * ALIGN) for r in range(self.world)]
            b.cut.append(b.numel)
        rcur = [0] * self.world
        for b in self.buckets:
            for r in range(self.world):
                b.rd_off.append(rcur[r])
                rcur[r] += b.cut[r + 1] - b.cut[r]
        self._rd_len = max(max(rcur) if rcur else 0, ALIGN)
        self._owned_units = [su for su in self.sunits if su.owner == self.rank]

    @torch.no_grad()
    def _materialize(self, model, dest, meta, init="serial"):
        """Give every parameter its storage and its value: from the model itself, or (meta model)
        from the streamed initialisation, one component at a time."""
        if meta:
            from ..models.init_stream import named_device_initial_tensors, named_initial_tensors
            source = (named_initial_tensors(model.cfg) if init == "serial"
                      else named_device_initial_tensors(model.cfg, self.device))
        else:
            source = [(n, p.detach()) for n, p in model.named_parameters() if n in dest]
        modules = dict(model.named_modules())
        filled = set()

        def place(p, t):
            if p.is_meta:  # a meta tensor cannot take storage through .data: swap the tensor in place
                torch.utils.swap_tensors(p, torch.nn.Parameter(t, requires_grad=p.requires_grad))
            else:
                p.data = t

        for name, value in source:
            if name in dest:
                p, target = dest[name]
                if target is not None:
                    target.copy_(value)
                    place(p, target)
                else:
                    place(p, self._zero.expand(p.shape))
                    p._ttb_remote = True
                filled.add(name)
            elif meta:  # buffers and frozen parameters: replicated as they are
                mod_name, _, attr = name.rpartition(".")
                mod = modules[mod_name]
                if attr in mod._parameters:
                    place(mod._parameters[attr], value.to(self.device, copy=True))
                elif attr in mod._buffers:
                    mod._buffers[attr] = value.to(self.device, copy=True)
        missing = set(dest) - filled
        if missing:
            raise ValueError(f"parameters without an initial value: {sorted(missing)[:5]}")
        if meta:
            left = [n for n, t in list(model.named_parameters()) + list(model.named_buffers()) if t.is_meta]
            if left:
                raise ValueError(f"model state left on the meta device: {left[:5]}")

    # ------------------------------------------------------------------ symmetric memory
    def _init_symmetric(self, device, dtype):
        # plain peer mappings only: these kernels use ordinary loads and stores, never multimem
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        import torch.distributed._symmetric_memory as symm_mem
        group = self.group if self.group is not None else dist.group.WORLD
        enable = getattr(symm_mem, "enable_symm_mem_for_group", None)
        if enable is not None:
            enable(group.group_name)
        n = self._flat_len
        self.grad_flat = symm_mem.empty(n, dtype=dtype, device=device)
        self.param_flat = symm_mem.empty(n, dtype=dtype, device=device)
        self.grad_flat.zero_()
        self.param_flat.zero_()
        hg = symm_mem.rendezvous(self.grad_flat, group)
        hp = symm_mem.rendezvous(self.param_flat, group)
        handles = [hg, hp]
        self._gptrs = [int(x) for x in hg.buffer_ptrs]
        self._pptrs = [int(x) for x in hp.buffer_ptrs]
        self._pads = [int(x) for x in hg.signal_pad_ptrs]
        self.stage = None
        if not self.shard_params:
            self.sp_param = torch.zeros(self.s_shard, device=device, dtype=dtype)
        else:
            self.sp_param = symm_mem.empty(self.s_shard, dtype=dtype, device=device)
            self.sp_param.zero_()
            hs = symm_mem.rendezvous(self.sp_param, group)
            self._spptrs = [int(x) for x in hs.buffer_ptrs]
            self.stage = symm_mem.empty(2 * self.max_bucket, dtype=torch.float32, device=device)
            self.stage.zero_()
            ht = symm_mem.rendezvous(self.stage, group)
            self._stptrs = [int(x) for x in ht.buffer_ptrs]
            # this rank's reduction slices of every block, accumulated over the micro-batches
            self.rd_grad = symm_mem.empty(self._rd_len, dtype=torch.float32, device=device)
            self.rd_grad.zero_()
            hr = symm_mem.rendezvous(self.rd_grad, group)
            self._rdptrs = [int(x) for x in hr.buffer_ptrs]
            handles.append(hr)
            # the per-block reductions run on their own stream, beside the next block's backward,
            # with their own barrier pads and epochs (independent of the compute-stream barriers)
            self._stpads = [int(x) for x in ht.signal_pad_ptrs]
            self._st_epoch = 0
            self._comm = torch.cuda.Stream(device)
            self._slot_free = [None, None]  # event: every owner has read the slot (None: never used)
            handles += [hs, ht]
            if self.fused_gather:
                handles.append(self._init_row_shards(device))
        self._handles = handles
        self._epoch = 0

    def _init_row_shards(self, device):
        """Symmetric bf16 buffer of this rank's row slice of every sharded group (same offsets on every
        rank), the staging window, and each group's gather description."""
        from .gather import GatheredWeight, GatherWindow, row_cuts
        woff, largest = 0, 0
        for su in self.sunits:
            su.rows, su.cols = sum(su.group.rows), su.group.d_in
            su.cuts = row_cuts(su.rows, self.world)
            su.woff = woff
            woff += _aligned(max(b - a for a, b in zip(su.cuts, su.cuts[1:])) * su.cols)
            largest = max(largest, su.rows * su.cols)
        handle = None
        if self.peer:
            import torch.distributed._symmetric_memory as symm_mem
            group = self.group if self.group is not None else dist.group.WORLD
            self.wshard = symm_mem.empty(max(woff, ALIGN), dtype=torch.bfloat16, device=device)
            handle = symm_mem.rendezvous(self.wshard, group)
            self._wsptrs = [int(x) for x in handle.buffer_ptrs]
        else:  # one rank: its shard is every row, read from its own memory
            self.wshard = torch.empty(max(woff, ALIGN), dtype=torch.bfloat16, device=device)
            self._wsptrs = [self.wshard.data_ptr()]
        slots = int(os.environ.get("TTB_GATHER_SLOTS", "8"))
        self.window = GatherWindow(device, slots, (largest + 127) // 128 * 128)
        for su in self.sunits:
            su.group._gather = GatheredWeight(self.window, su.rows, su.cols, su.cuts,
                                              [base + 2 * su.woff for base in self._wsptrs])
        return handle

    def _build_gather_plan(self):
        """Copy segments of the fused all-gather: every replicated unit from its owner's buffer into
        the local one (own units are not copied), plus the bf16 cache of every weight group
        (sharded groups: straight from the owner's master)."""
        from ..ops._ext import lib
        rows, owners, max_n = [], [], 0
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
            owners.append(r)
            max_n = max(max_n, n4)
        for su in self.sunits:
            if self.fused_gather:  # this rank's rows of the group, from the owner's master
                lo, hi = su.cuts[self.rank], su.cuts[self.rank + 1]
                if hi > lo:
                    rows.append((self._spptrs[su.owner] + 4 * (su.goff + lo * su.cols), 0,
                                 self.wshard.data_ptr() + 2 * su.woff, (hi - lo) * su.cols))
                    owners.append(su.owner)
                    max_n = max(max_n, (hi - lo) * su.cols)
                continue
            cache = su.group.bf16()
            assert cache.numel() == su.n and su.n % 4 == 0
            rows.append((self._spptrs[su.owner] + 4 * su.goff, 0, cache.data_ptr(), su.n))
            owners.append(su.owner)
            max_n = max(max_n, su.n)
        # the kernel takes segments roughly in list order; starting each rank at the next rank's units
        # (and ending at its own) spreads the pulls over every owner at once instead of every rank
        # reading owner 0 first
        order = sorted(range(len(rows)), key=lambda i: ((owners[i] - self.rank - 1) % self.world, i))
        rows = [rows[i] for i in order]
        self._segs = torch.tensor(rows, dtype=torch.int64).to(self.param_flat.device) if rows else None
        self._seg_max = max_n
        self._lib = lib
        # owned units' gradients from the reduction slices: piece [x0, x1) of a unit's staging range
        # held by rank q sits at rd_off(q) + x0 - cut(q) of q's rd_grad
        segs, seg_max = [], 0
        if self.shard_params:
            sp = self.sp_grad.data_ptr()
            for su in self._owned_units:
                b = self.buckets[su.bucket]
                u0, u1 = su.stage_off, su.stage_off + _aligned(su.n)
                for q in range(self.world):
                    x0, x1 = max(u0, b.cut[q]), min(u1, b.cut[q + 1])
                    if x1 > x0:
                        segs.append((self._rdptrs[q] + 4 * (b.rd_off[q] + x0 - b.cut[q]),
                                     sp + 4 * (su.goff + x0 - u0), 0, x1 - x0))
                        seg_max = max(seg_max, x1 - x0)
        self._rd_segs = torch.tensor(segs, dtype=torch.int64).to(self.param_flat.device) if segs else None
        self._rd_seg_max = seg_max

    def _stage_barrier(self):
        self._st_epoch += 1
        self._lib().peer_barrier(self._stpads, self.rank, self._st_epoch, BARRIER_LIMIT_CYCLES)

    def _barrier(self, limit=None):
        self._epoch += 1
        if limit is None:
            self._lib().peer_barrier(self._pads, self.rank, self._epoch)
        else:
            self._lib().peer_barrier(self._pads, self.rank, self._epoch, limit)

    def _name(self, p):
        return self._names.get(id(p), "?")

    # ------------------------------------------------------------------ ownership
    def owned_params(self) -> list[torch.Tensor]:
        own = [p for _, _, params, _, _, r in self.units if r == self.rank for p in params]
        return own + [p for su in self._owned_units for p in su.params]

    def owned_ids(self) -> set[int]:
        return {id(p) for p in self.owned_params()}

    def region(self, flat: torch.Tensor) -> torch.Tensor:
        start = self._rstart[self.rank]
        return flat[start:start + self._rlen[self.rank]]

    def sharded_names(self) -> set[str]:
        """Parameters held only by their owner (parameter-sharded mode)."""
        return {n for su in self.sunits for n in su.names}

    def owned_sharded_state(self) -> dict:
        return {n: p.detach() for su in self._owned_units for n, p in zip(su.names, su.params)}

    def replicated_state(self) -> dict:
        """The model state every rank holds identically between steps."""
        skip = self.sharded_names()
        return {k: v for k, v in self.model.state_dict().items() if k not in skip}

    # ------------------------------------------------------------------ per-layer gradient reduction
    def _stage_view(self, su):
        b = self.buckets[su.bucket]
        base = (b.index % 2) * self.max_bucket + su.stage_off
        return self.stage[base:base + su.n].view(sum(su.group.rows), su.group.d_in)

    def sink(self, su, compute):
        """Weight-gradient GEMM of a sharded group: into the block's staging slot (overwrite)."""
        if self.peer:  # the slot's previous bucket must have been read by every owner
            ev = self._slot_free[self.buckets[su.bucket].index % 2]
            if ev is not None:
                torch.cuda.current_stream().wait_event(ev)
        compute(self._stage_view(su), 0.0)
        su.pending = 0
        self._unit_ready(su)
        return [None] * len(su.params)

    def _param_ready(self, su, p):
        su.pending -= 1
        if su.pending == 0:
            self._unit_ready(su)

    def _unit_ready(self, su):
        b = self.buckets[su.bucket]
        b.ready += 1
        if b.ready == len(b.units):
            self._reduce_bucket(b)

    def _reduce_bucket(self, b, missing=()):
        """Add the rank-summed gradient of bucket ``b`` into the owners' accumulators."""
        lo, n, goff = b.own_off[self.rank], b.own_n[self.rank], b.own_goff[self.rank]
        if self._cache_mode:
            slot = (b.index % 2) * self.max_bucket
            for su in missing:  # units without a gradient this micro-batch contribute zeros
                self._stage_view(su).zero_()
            if self.peer:
                # on the communication stream, after this rank's GEMMs of the bucket: barrier (every
                # rank has written its slot), pull-accumulate the owned range, barrier (every owner
                # has read it); the compute stream waits for that before it writes the slot again
                written = torch.cuda.Event()
                written.record()
                lo_r, hi_r = b.cut[self.rank], b.cut[self.rank + 1]
                rd = b.rd_off[self.rank]
                with torch.cuda.stream(self._comm):
                    self._comm.wait_event(written)
                    self._stage_barrier()
                    if hi_r > lo_r:
                        self._lib().rs_accumulate(self._stptrs, slot + lo_r, self.rd_grad[rd:rd + hi_r - lo_r],
                                                  PULL_BLOCKS)
                    self._stage_barrier()
                    free = torch.cuda.Event()
                    free.record(self._comm)
                self._slot_free[b.index % 2] = free
            else:
                flat = self.stage[slot:slot + b.numel]
                if self.world > 1:
                    dist.all_reduce(flat, group=self.group)
                if n:
                    self.sp_grad[goff:goff + n] += flat[lo:lo + n]
        else:
            flat = torch.zeros(b.numel, device=self.device, dtype=self.dtype)
            for su in b.units:
                pos = su.stage_off
                for p in su.params:
                    if p.grad is not None:
                        flat[pos:pos + p.numel()].copy_(p.grad.reshape(-1))
                        p.grad = None
                    pos += p.numel()
            if self.world > 1:
                dist.all_reduce(flat, group=self.group)
            if n:
                self.sp_grad[goff:goff + n] += flat[lo:lo + n]
        b.ready = 0
        for su in b.units:
            su.pending = len(su.params)

    def after_backward(self):
        """End of one micro-batch's backward: reduce the buckets whose units did not all receive a
        gradient (e.g. an ablated branch), with zeros for the missing ones, in bucket order.  The
        model structure decides which units those are, so every rank reduces the same buckets."""
        if not self.shard_params:
            return
        for b in self.buckets:
            if b.ready:
                self._reduce_bucket(b, [su for su in b.units if su.pending])

    # ------------------------------------------------------------------ step phases
    def zero_grad(self):
        """Zero the gradient buffers and attach every replicated parameter's ``.grad`` view
        (backward accumulates); sharded parameters receive their gradient at the reduction."""
        self.grad_flat.zero_()
        for kind, obj, params, off, n, _ in self.units:
            pos = off
            for p in params:
                p.grad = self.grad_flat[pos:pos + p.numel()].view_as(p)
                pos += p.numel()
        if self.shard_params:
            self.sp_grad.zero_()
            if self.peer:
                self.rd_grad.zero_()
            for su in self.sunits:
                for p in su.params:
                    p.grad = None
                su.pending = len(su.params)
            for b in self.buckets:
                b.ready = 0

    def reduce_gradients(self):
        """Sum gradients over ranks; afterwards this rank's region holds its owned units' sums
        (sharded units were reduced layer by layer during backward)."""
        if self.shard_params:
            if self.peer:
                # the per-block reductions have landed in every rank's rd_grad: owners gather the
                # pieces of their units from the slice holders, then no rank zeroes rd_grad early
                torch.cuda.current_stream().wait_stream(self._comm)
                self._stage_barrier()
                if self._rd_segs is not None:
                    self._lib().ag_pull_cast(self._rd_segs, self._rd_seg_max)
                self._stage_barrier()
            for su in self._owned_units:
                pos = su.goff
                for p in su.params:
                    p.grad = self.sp_grad[pos:pos + p.numel()].view(p.shape)
                    pos += p.numel()
        if self.world == 1:
            return
        self._sq = None
        if self.peer:
            self._barrier()  # every rank's backward has finished writing its buffer
            mine = self.region(self.grad_flat)
            if mine.numel():
                self._sq = self._lib().rs_reduce_sq(self._gptrs, self._rstart[self.rank], mine).sum()
            else:
                self._sq = torch.zeros((), device=self.device, dtype=torch.float64)
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
        if self.shard_params and self.s_shard:
            sq = sq + torch.linalg.vector_norm(self.sp_grad).double().square()
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        return sq

    def clip_coefficient(self, max_norm: float) -> tuple[torch.Tensor, torch.Tensor]:
        """(pre-clip global norm, clip coefficient) as device fp32 scalars; the gradients are left
        as they are for an optimizer that applies the coefficient while it reads them."""
        norm = self.grad_norm_sq().sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0).to(torch.float32).reshape(1)
        return norm.float(), coef

    def clip_(self, max_norm: float) -> torch.Tensor:
        """Scale the owned gradients so the global norm is at most ``max_norm`` (the rule of
        torch.nn.utils.clip_grad_norm_); returns the pre-clip global norm (fp32, on the device)."""
        norm = self.grad_norm_sq().sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0).to(self.grad_flat.dtype)
        self.region(self.grad_flat).mul_(coef)
        if self.shard_params:
            self.sp_grad.mul_(coef)
        return norm.float()

    @torch.no_grad()
    def gather_params(self):
        """Bring every rank the owners' updated parameters (sharded units: their bf16 caches, or the
        compute copies off the fused path)."""
        if self.peer:
            self._barrier()  # every owner has updated its region
            if self._segs is not None:
                self._lib().ag_pull_cast(self._segs, self._seg_max)
            for kind, obj, *_ in self.units:
                if kind == "group":
                    obj._key = obj._version_key()  # the caches were written from the gathered values
            if self.fused_gather:
                self.window.invalidate()
                self._barrier()  # every rank's row shards are written before any GEMM gathers from them
            return
        if self.world > 1:
            if self.backend == "nccl":
                dist.all_gather_into_tensor(self.param_flat, self.region(self.param_flat), group=self.group)
            else:
                for r, global_rank in enumerate(self._ranks):
                    dist.broadcast(self.param_flat[r * self.shard:(r + 1) * self.shard], src=global_rank,
                                   group=self.group)
        if not self.shard_params:
            return
        if self.fused_gather:  # one rank: its row shard of every group is all of the group's rows
            for su in self.sunits:
                self.wshard[su.woff:su.woff + su.n].view(su.rows, su.cols).copy_(
                    torch.cat([p.detach().reshape(-1, su.cols) for p in su.params]))
            self.window.invalidate()
            return
        for su in self.sunits:
            src = self._ranks[su.owner]
            if self._cache_mode:
                grp = su.group
                if su.owner == self.rank or grp._cache is None:
                    grp._shard = None  # build from the master (owner) or allocate (others)
                    cache = grp.bf16()
                    grp._shard = (self, su)
                if self.world > 1:
                    dist.broadcast(grp._cache, src=src, group=self.group)
            elif self.world > 1:
                if su.owner == self.rank:
                    flat = torch.cat([p.detach().reshape(-1) for p in su.params])
                else:
                    flat = torch.empty(su.n, device=self.device, dtype=self.dtype)
                dist.broadcast(flat, src=src, group=self.group)
                if su.owner != self.rank:
                    pos = 0
                    for p in su.params:
                        p.copy_(flat[pos:pos + p.numel()].view(p.shape))
                        pos += p.numel()

    # ------------------------------------------------------------------ full state
    def full_state_dict(self, dst: int | None = 0) -> dict | None:
        """The complete model state on CPU, assembled from the owners (collective; every rank
        calls).  Returned on rank ``dst`` (every rank when ``dst`` is None), None elsewhere."""
        state = {k: v.detach().cpu().clone() for k, v in self.replicated_state().items()}
        for su in self.sunits:
            if su.owner == self.rank:
                flat = torch.cat([p.detach().reshape(-1) for p in su.params])
            else:
                flat = torch.empty(su.n, device=self.device, dtype=self.dtype)
            if self.world > 1:
                dist.broadcast(flat, src=self._ranks[su.owner], group=self.group)
            if dst is None or self.rank == dst:
                pos = 0
                for p, name in zip(su.params, su.names):
                    state[name] = flat[pos:pos + p.numel()].view(p.shape).cpu().clone()
                    pos += p.numel()
        if dst is not None and self.rank != dst:
            return None
        model_keys = list(self.model.state_dict().keys())
        return {k: state[k] for k in model_keys if k in state}

    @torch.no_grad()
    def load_owned_sharded(self, state: dict):
        for su in self._owned_units:
            for p, name in zip(su.params, su.names):
                p.copy_(state[name])
