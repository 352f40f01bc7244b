"""The training-step engine: the public call a user (or a trainer) makes for one optimizer update.

``TrainEngine.step(idx, doc_ids, targets)`` takes this rank's share of a global batch (CPU --
ideally pinned -- or CUDA tensors), splits it into micro-batches, copies each to the device
(non-blocking), runs forward/backward on the fused sm_100a path with the reference's
loss-normalization contract (every rank back-propagates ``local_sum / global_valid_targets``),
sums gradients across ranks (one reduce-scatter onto the owning ranks), clips the global norm,
steps the optimizer on the owned parameters and all-gathers the updated parameters.  It returns
the step's summed loss and valid-target count as device tensors (no host synchronisation).

``step`` is built on three primitives that trainers with their own batching use directly:
``begin_update`` (zero the gradients), ``forward_loss`` / ``backward`` per micro-batch, and
``finish_update``, which can divide the accumulated gradients by the update's target count
afterwards (the serial trainer's contract: sum the micro-batch losses, then divide) instead of
scaling each micro-batch's loss beforehand.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .config import Config
from .models.model import TensorLM
from .optim import make_optimizer
from .parallel.sharded import ShardedDataParallel


class TrainEngine:
    def __init__(self, cfg: Config, device="cuda", micro_batch: int = 8, model: TensorLM | None = None,
                 optimizer=None, group=None, grad_clip: float | None = None, shard_params: bool | None = None,
                 init: str = "serial", recompute_blocks: int | None = None):
        """``shard_params``: keep fp32 weights, gradients and optimizer state only on their owner
        rank (None: when ``TTB_SHARD_PARAMS=1`` or when the replicated layout would not fit the
        device; see models.shapes.needs_parameter_sharding).  A sharded engine builds its model
        itself from the streamed serial initialisation unless ``model`` is given (``init="device"``:
        the same distributions drawn on the device, for throughput runs).  ``recompute_blocks``
        (or ``TTB_RECOMPUTE_BLOCKS``): under activation checkpointing, recompute only the first this
        many blocks and keep the others' activations (selective recompute where memory allows);
        ``"auto"`` picks the count from the capacity plan and this GPU's memory."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.micro_batch = int(micro_batch)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if shard_params is None:
            from .models.shapes import needs_parameter_sharding
            shard_params = needs_parameter_sharding(cfg.model, self.world, self.device)
        self.shard_params = bool(shard_params)
        if model is None:
            if self.shard_params:
                with torch.device("meta"):
                    model = TensorLM(cfg.model)
            else:
                model = TensorLM(cfg.model).to(self.device)
        self.model = model
        self.model.train()
        if recompute_blocks is None and os.environ.get("TTB_RECOMPUTE_BLOCKS"):
            recompute_blocks = os.environ["TTB_RECOMPUTE_BLOCKS"]
        # "auto" is resolved at the first micro-batch, when the tokens per micro-batch are known
        self._recompute_auto = recompute_blocks == "auto"
        if recompute_blocks is not None and not self._recompute_auto:
            self.model.recompute_blocks = int(recompute_blocks)
        self.grad_clip = cfg.train.grad_clip if grad_clip is None else grad_clip
        self.fused = self.device.type == "cuda" and self.model.fused_path_supported()[0]
        # flat gradient/parameter buffers: needed by the fused path and by every multi-rank run
        self.dp = (ShardedDataParallel(self.model, self.device, group, fused=self.fused,
                                       shard_params=self.shard_params, init=init)
                   if self.fused or self.world > 1 or self.shard_params else None)
        if optimizer is None:
            only = self.dp.owned_ids() if self.dp is not None and (self.world > 1 or self.shard_params) else None
            optimizer = make_optimizer(self.model, cfg.train, only=only)
        elif callable(optimizer) and not isinstance(optimizer, torch.optim.Optimizer):
            optimizer = optimizer(self.model)  # built after the parameters moved into the flat buffers
        self.optimizer = optimizer
        self.last_grad_norm = None
        # optional per-phase device timing: a list that receives, per step, the (phase, CUDA event) pairs
        # recorded at the end of each phase
        self.phase_events: list | None = None

    def _resolve_auto_recompute(self, tokens: int):
        """Blocks to recompute so that the capacity plan with the rest kept fits 92 % of this GPU
        (``recompute_blocks="auto"``; resolved once, at the first micro-batch of ``tokens`` tokens)."""
        self._recompute_auto = False
        if self.device.type != "cuda" or not self.cfg.model.activation_checkpointing:
            return
        from .models.shapes import blocks_to_recompute
        total = torch.cuda.get_device_properties(self.device).total_memory
        self.model.recompute_blocks = blocks_to_recompute(
            self.cfg.model, gpus=self.world, micro_tokens_per_gpu=tokens, device_bytes=total,
            shard_params=self.shard_params, optimizer=self.cfg.train.optimizer)

    def _mark(self, marks, name):
        if marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

    def _to_device(self, t):
        if t.device == self.device:
            return t
        return t.to(self.device, non_blocking=True)

    def zero_grad(self):
        if self.dp is not None:
            self.dp.zero_grad()
        else:
            self.optimizer.zero_grad(set_to_none=True)

    # ------------------------------------------------------------------ primitives
    def begin_update(self):
        self.zero_grad()

    def forward_loss(self, idx, doc_ids, targets):
        """One micro-batch's forward: (summed loss, valid-target count) on the device."""
        if self._recompute_auto:
            self._resolve_auto_recompute(idx.numel())
        i, d, t = (self._to_device(x) for x in (idx, doc_ids, targets))
        _, loss, n = self.model(i, d, t, reduction="sum")
        return loss, n

    def backward(self, objective):
        objective.backward()
        if self.dp is not None:
            self.dp.after_backward()

    def _clip(self, error_if_nonfinite: bool):
        """Clip norm and, for optimizers that apply it while reading gradients, the coefficient."""
        if not (self.grad_clip and self.grad_clip > 0):
            return None, None
        if self.dp is not None and getattr(self.optimizer, "accepts_grad_scale", False):
            norm, scale = self.dp.clip_coefficient(self.grad_clip)
        elif self.dp is not None:
            norm, scale = self.dp.clip_(self.grad_clip), None
        else:
            params = (self.model.parameters() if error_if_nonfinite
                      else [p for p in self.model.parameters() if p.grad is not None])
            return torch.nn.utils.clip_grad_norm_(params, self.grad_clip, error_if_nonfinite=error_if_nonfinite,
                                                  foreach=None if error_if_nonfinite else True), None
        if error_if_nonfinite and not bool(torch.isfinite(norm)):
            raise RuntimeError(f"The total norm of gradients is non-finite ({float(norm)}), so it cannot be clipped")
        return norm, scale

    def finish_update(self, *, divide_by: float | None = None, error_if_nonfinite: bool = False, marks=None):
        """Sum gradients across ranks, divide them by ``divide_by`` if given, clip, step the optimizer
        and bring every rank the updated parameters.  Returns the pre-clip gradient norm."""
        if self.dp is not None:
            self.dp.reduce_gradients()
        self._mark(marks, "reduce_gradients")
        if divide_by is not None:
            grads = [p.grad for p in self.model.parameters() if p.grad is not None]
            torch._foreach_div_(grads, float(divide_by))
        self.last_grad_norm, scale = self._clip(error_if_nonfinite)
        self._mark(marks, "clip")
        if scale is not None:
            self.optimizer.step(grad_scale=scale)
        else:
            self.optimizer.step()
        self._mark(marks, "optimizer")
        if self.dp is not None:
            self.dp.gather_params()
        self._mark(marks, "gather_params")
        return self.last_grad_norm

    def forward_backward(self, idx, doc_ids, targets, inv_count):
        """Accumulate gradients of sum(loss) * inv_count over micro-batches; returns the loss sum."""
        loss_total = torch.zeros((), device=self.device, dtype=torch.float32)
        rows = idx.shape[0]
        for s in range(0, rows, self.micro_batch):
            e = min(rows, s + self.micro_batch)
            loss, _ = self.forward_loss(idx[s:e], doc_ids[s:e], targets[s:e])
            self.backward(loss * inv_count)
            loss_total += loss.detach().float()
        return loss_total

    def step(self, idx, doc_ids, targets, lr_multiplier: float | None = None):
        """One optimizer update on this rank's rows.  Returns (loss_sum, global_count) on the device."""
        if lr_multiplier is not None:
            for g in self.optimizer.param_groups:
                g["lr"] = g.get("base_lr", g["lr"]) * lr_multiplier
        marks = [] if self.phase_events is not None and self.device.type == "cuda" else None
        self._mark(marks, "start")
        self.begin_update()
        # valid-target count: counted on the host side of the copy, summed over ranks on the device
        local = (targets != -100).sum()
        count = local.to(self.device, non_blocking=True).to(torch.int64)
        if self.world > 1:
            dist.all_reduce(count, group=self.group)
        inv = 1.0 / count.clamp_min(1).to(torch.float32)
        loss_sum = self.forward_backward(idx, doc_ids, targets, inv)
        self._mark(marks, "forward_backward")
        if self.world > 1:
            dist.all_reduce(loss_sum, group=self.group)
        self.finish_update(marks=marks)
        if marks is not None:
            self.phase_events.append(marks)
        return loss_sum, count

    def phase_times_ms(self) -> dict:
        """Mean device milliseconds per step of each phase recorded in ``phase_events`` (call after a
        device synchronise); the phases are consecutive intervals on the compute stream."""
        out: dict[str, float] = {}
        steps = self.phase_events or []
        for marks in steps:
            for (_, a), (name, b) in zip(marks, marks[1:]):
                out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return {k: round(v / len(steps), 3) for k, v in out.items()} if steps else {}
