"""Stability instrumentation of a training run: its policy, the per-batch score bounds that feed
QK-clip, and a fixed probe row for diagnostics.

* ``StabilityPolicy`` reads and checks the four ``train`` fields involved: how often to record
  stability statistics, the QK-clip threshold and cadence, and where clip maxima come from
  ("probe" or "batch_bound").
* ``BatchScoreBounds`` collects, over the micro-batches of one update, the score bounds each
  polynomial attention layer records in its forward; the update's maximum goes to metrics and the
  last micro-batch's per-head bounds drive a ``batch_bound`` clip.  The maximum covers padding and
  unscored positions and bounds the scores before the update, not after it.
* ``TrainingStabilityProbe`` holds the first row (at most 512 tokens) of an independent train-split
  sampler, so it never consumes the training stream, and runs statistics or a probe clip on it
  between updates with module modes, norm statistics collection, score-bound recording and every
  RNG restored afterwards.

Behaviour as the reference's (tnlm/training_stability.py:15-196).
"""
from __future__ import annotations

import math
import random
import time
from contextlib import contextmanager
from dataclasses import dataclass

import numpy as np
import torch

from .models.normalization import lagged_modules, taper_modules

OPTIMIZER_STATE_POLICY = "moments and step counters unchanged"
PROBE_MAX_CONTEXT = 512


@dataclass(frozen=True)
class StabilityPolicy:
    stability_every: int
    clip_tau: float
    clip_every: int
    clip_source: str

    @classmethod
    def from_config(cls, cfg) -> "StabilityPolicy":
        t = cfg.train
        every = getattr(t, "stability_every_steps", 0)
        if isinstance(every, bool) or not isinstance(every, int) or every < 0:
            raise ValueError("train.stability_every_steps must be an integer >= 0")
        source = getattr(t, "qk_clip_source", "probe")
        if type(source) is not str or source not in ("probe", "batch_bound"):
            raise ValueError("train.qk_clip_source must be 'probe' or 'batch_bound'")
        if source == "batch_bound" and cfg.model.attention == "softmax":
            raise ValueError("batch_bound score recording needs polynomial attention")
        tau = getattr(t, "qk_clip_tau", 0.0)
        if type(tau) not in (int, float) or not math.isfinite(tau) or tau < 0:
            raise ValueError("train.qk_clip_tau must be finite and nonnegative")
        cadence = getattr(t, "qk_clip_every_steps", 0)
        if type(cadence) is not int or cadence < 0 or (tau > 0 and cadence == 0):
            raise ValueError("train.qk_clip_every_steps must be a nonnegative integer, positive when clipping is on")
        if tau > 0 and cfg.model.normalization == "spectral_rms":
            raise ValueError("QK-clip does not support spectral_rms models")
        return cls(every, float(tau), cadence, source)

    @property
    def clipping(self) -> bool:
        return self.clip_tau > 0

    def needs_probe(self) -> bool:
        return bool(self.stability_every) or (self.clipping and self.clip_source == "probe")


def sanitize_finite(value, root: str) -> tuple:
    """(copy of ``value`` with non-finite floats replaced by None, the paths that were replaced)."""
    bad: list[str] = []

    def walk(v, path):
        if isinstance(v, dict):
            return {k: walk(x, f"{path}.{k}") for k, x in v.items()}
        if isinstance(v, (list, tuple)):
            return [walk(x, f"{path}[{i}]") for i, x in enumerate(v)]
        if isinstance(v, (float, np.floating)):
            if math.isfinite(v):
                return float(v)
            bad.append(path)
            return None
        return v
    return walk(value, root), bad


def _require_finite_clip(stats: dict) -> None:
    _, bad = sanitize_finite(stats, "qk_clip")
    if bad:
        raise FloatingPointError("QK-clip produced non-finite values at " + ", ".join(bad))


class BatchScoreBounds:
    """Attention-score bounds of one optimizer update, taken from the training forwards themselves.

    Each micro-batch's forward records, per layer and score factor (S1, and S2 for two-factor
    attention), every head's bound max|q|*max|k|/sqrt(dk) (the QKV GEMM's epilogue emits the row
    norms on the fused path).  The update's diagnostic is the largest bound over all its micro-batches
    (NaN, which aborts the update, once any bound is negative); QK-clip uses the per-head bounds of
    the update's last micro-batch, as the reference does (tnlm/training_stability.py:57-130).  The
    bounds are snapshotted after each forward because the kernels reuse their output buffers and an
    activation-checkpointing backward would record again."""

    def __init__(self, model, cfg):
        from .qk_clip import set_score_bound_recording
        self.model = model
        self.enabled = StabilityPolicy.from_config(cfg).clip_source == "batch_bound"
        self._factors = [("S1", "S2") if hasattr(blk.attn, "q2") else ("S1",) for blk in model.blocks]
        self.top: torch.Tensor | None = None   # device scalar over the update so far
        self.last: list[dict] | None = None    # per layer {factor: (H,)} of the latest micro-batch
        if self.enabled:
            set_score_bound_recording(model, True)

    def begin_update(self) -> None:
        self.top = self.last = None

    def _snapshot(self) -> tuple[torch.Tensor, list[dict]]:
        """One stacked copy of every recorded bound, and per-layer views into it."""
        from .qk_clip import score_bounds
        heads, flat, keys = self.model.cfg.heads, [], []
        for layer, (expected, got) in enumerate(zip(self._factors, score_bounds(self.model))):
            if set(got) != set(expected):
                raise ValueError(f"layer {layer} recorded no or unexpected score-bound factors")
            for factor in expected:
                b = got[factor]
                if not torch.is_tensor(b) or b.shape != (heads,):
                    raise ValueError(f"layer {layer} {factor}: a score bound must be a ({heads},) tensor")
                flat.append(b.detach())
                keys.append((layer, factor))
        if not flat:
            raise ValueError("no polynomial attention layer recorded score bounds")
        stacked = torch.stack(flat)
        views = [{} for _ in self.model.blocks]
        for row, (layer, factor) in zip(stacked, keys):
            views[layer][factor] = row
        return stacked, views

    def observe(self) -> None:
        """Fold the micro-batch just run into the update (device-side, no host synchronisation)."""
        if not self.enabled:
            return
        stacked, self.last = self._snapshot()
        worst = torch.where((stacked < 0).any(), stacked.new_tensor(float("nan")), stacked.max())
        self.top = worst if self.top is None else torch.maximum(self.top, worst)

    def finish_update(self) -> float:
        """The update's largest bound (the one host read); raises when it is missing or invalid."""
        if not self.enabled:
            return 0.0
        if self.top is None:
            raise ValueError("this update recorded no score bounds")
        value = float(self.top)
        if not (math.isfinite(value) and value >= 0):
            raise FloatingPointError("a score bound was non-finite or negative; the update is aborted")
        return value

    def reduce_last(self, all_reduce_max_) -> None:
        """Data-parallel ranks each ran their own last micro-batch, so their recorded per-head bounds
        differ; clipping from them would rescale the replicated Q/K weights differently on each rank.
        This replaces them with their maximum over the ranks (``all_reduce_max_`` reduces a flat fp64
        CPU tensor in place), a bound on the scores of every rank's last micro-batch, so every rank
        clips by the same factors.  A rank that ran no micro-batch contributes zeros (bounds are
        nonnegative)."""
        heads = self.model.cfg.heads
        layout = [(layer, f) for layer, factors in enumerate(self._factors) for f in factors]
        flat = torch.zeros(len(layout) * heads, dtype=torch.float64)
        if self.last is not None:
            for k, (layer, f) in enumerate(layout):
                flat[k * heads:(k + 1) * heads] = self.last[layer][f].detach().to("cpu", torch.float64)
        all_reduce_max_(flat)
        self.last = [{} for _ in self.model.blocks]
        for k, (layer, f) in enumerate(layout):
            self.last[layer][f] = flat[k * heads:(k + 1) * heads]

    def clip(self, tau) -> dict:
        """Rescale every head over ``tau`` by the last micro-batch's bounds (after checking the update's)."""
        from .qk_clip import qk_clip_from_bounds_
        self.finish_update()
        if self.last is None:
            raise ValueError("no last-micro-batch score bounds to clip from")
        for blk, bounds in zip(self.model.blocks, self.last):
            blk.attn.last_score_bound = bounds
        t0 = time.monotonic()
        stats = qk_clip_from_bounds_(self.model, tau)
        _require_finite_clip(stats)
        return {**stats, "seconds": time.monotonic() - t0, "optimizer_state_policy": OPTIMIZER_STATE_POLICY}


class TrainingStabilityProbe:
    def __init__(self, cfg, device):
        from .data import PackedSampler, batch_hash
        self.device = torch.device(device)
        data = cfg.raw["data"]
        context = min(data.get("context", 512), PROBE_MAX_CONTEXT)
        sampler = PackedSampler(data["manifest"], split="train", batch_size=1, context=context, seed=cfg.train.seed)
        batch = sampler.next_batch()
        self.identity = {"batch_sha256": batch_hash(batch), "manifest_sha256": sampler.manifest_hash,
                         "split": "train", "seed": cfg.train.seed, "context": context, "batch_size": 1}
        self.idx, self.doc = (t.to(self.device) for t in batch[:2])

    @contextmanager
    def _isolated(self, model):
        """Eval mode, no norm statistics, no score recording, forked RNGs; all restored on exit."""
        modes = [(m, m.training) for m in model.modules()]
        norms = [(m, m.collecting, m._valid) for m in lagged_modules(model) + taper_modules(model)]
        recorders = [(b.attn, b.attn.record_score_bound, b.attn.last_score_bound) for b in model.blocks]
        host_rngs = (random.getstate(), np.random.get_state())
        cuda = ([self.device.index if self.device.index is not None else torch.cuda.current_device()]
                if self.device.type == "cuda" else [])
        try:
            with torch.random.fork_rng(devices=cuda), torch.no_grad():
                model.eval()
                for attn, _, _ in recorders:
                    attn.record_score_bound = False
                for m, _, _ in norms:
                    m.collecting = False
                yield
                if self.device.type == "cuda":
                    torch.cuda.synchronize(self.device)  # the probe's time includes finishing it
        finally:
            for attn, on, last in recorders:
                attn.record_score_bound, attn.last_score_bound = on, last
            for m, training in modes:
                m.training = training
            for m, collecting, valid in norms:
                m.collecting, m._valid = collecting, valid
            random.setstate(host_rngs[0])
            np.random.set_state(host_rngs[1])

    def sample(self, model) -> dict:
        from .analysis import stability_stats
        t0 = time.monotonic()
        with self._isolated(model):
            stats = stability_stats(model, self.idx, self.doc)
        clean, bad = sanitize_finite(stats, "stats")
        return {"stats": clean, "probe": dict(self.identity), "seconds": time.monotonic() - t0,
                "nonfinite_paths": bad}

    def clip(self, model, tau) -> dict:
        from .qk_clip import qk_clip_
        t0 = time.monotonic()
        with self._isolated(model):
            stats = qk_clip_(model, self.idx, self.doc, tau)
        _require_finite_clip(stats)
        return {**stats, "probe": dict(self.identity), "seconds": time.monotonic() - t0,
                "optimizer_state_policy": OPTIMIZER_STATE_POLICY}
