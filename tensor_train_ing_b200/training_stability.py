"""Training-time stability instrumentation: config policy checks, per-batch score bounds used by
QK-clip, and a fixed probe row from an independent train sampler (reference
tnlm/training_stability.py:15-196)."""
from __future__ import annotations

import math
import random
import time

import numpy as np
import torch

from .models.normalization import lagged_modules, taper_modules


def stability_interval(cfg) -> int:
    value = getattr(cfg.train, "stability_every_steps", 0)
    if isinstance(value, bool) or not isinstance(value, int) or value < 0:
        raise ValueError("train.stability_every_steps must be an integer >= 0")
    return value


def qk_clip_source(cfg) -> str:
    source = getattr(cfg.train, "qk_clip_source", "probe")
    if type(source) is not str or source not in ("probe", "batch_bound"):
        raise ValueError("train.qk_clip_source must be probe or batch_bound")
    if source == "batch_bound" and cfg.model.attention == "softmax":
        raise ValueError("batch_bound recording requires polynomial attention")
    return source


def qk_clip_policy(cfg):
    qk_clip_source(cfg)
    tau = getattr(cfg.train, "qk_clip_tau", 0.0)
    every = getattr(cfg.train, "qk_clip_every_steps", 0)
    if type(tau) not in (int, float) or not math.isfinite(tau) or tau < 0:
        raise ValueError("train.qk_clip_tau must be finite and nonnegative")
    if type(every) is not int or every < 0 or (tau > 0 and every == 0):
        raise ValueError("train.qk_clip_every_steps must be a nonnegative integer, positive when clipping is enabled")
    if tau > 0 and cfg.model.normalization == "spectral_rms":
        raise ValueError("QK clipping does not support spectral models")
    return float(tau), every


def finite_json(value, path, nonfinite):
    if isinstance(value, dict):
        return {k: finite_json(v, f"{path}.{k}", nonfinite) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [finite_json(v, f"{path}[{i}]", nonfinite) for i, v in enumerate(value)]
    if isinstance(value, (float, np.floating)):
        if not math.isfinite(value):
            nonfinite.append(path)
            return None
        return float(value)
    return value


class BatchScoreBounds:
    """Per-update maximum of the recorded per-batch score bounds (over micro-batches, layers and
    factors), and clipping from the last micro-batch's bounds."""

    def __init__(self, model, cfg):
        from .qk_clip import set_score_bound_recording
        self.model = model
        self.enabled = qk_clip_source(cfg) == "batch_bound"
        self.maximum = None
        self.last = None
        if self.enabled:
            set_score_bound_recording(model, True)

    def begin_update(self):
        self.maximum = self.last = None

    def observe(self):
        if not self.enabled:
            return
        from .qk_clip import score_bounds
        snapshot = score_bounds(self.model)
        entries = []
        for layer, (blk, bounds) in enumerate(zip(self.model.blocks, snapshot)):
            expected = {"S1", "S2"} if hasattr(blk.attn, "q2") else {"S1"}
            if set(bounds) != expected:
                raise ValueError("missing or invalid polynomial score bounds")
            for name, bound in bounds.items():
                if not torch.is_tensor(bound) or bound.shape != (self.model.cfg.heads,):
                    raise ValueError("invalid score bound shape")
                entries.append((layer, name, bound.detach()))
        if not entries:
            raise ValueError("no polynomial score bounds were recorded")
        values = torch.cat([b for _, _, b in entries])
        mx = values.amax()
        mx = torch.where((values < 0).any(), mx.new_full((), float("nan")), mx)
        self.maximum = mx if self.maximum is None else torch.maximum(self.maximum, mx)
        heads = self.model.cfg.heads
        self.last = [{} for _ in snapshot]
        for k, (layer, name, _) in enumerate(entries):
            self.last[layer][name] = values[k * heads:(k + 1) * heads]

    def finish_update(self) -> float:
        if not self.enabled:
            return 0.0
        if self.maximum is None:
            raise ValueError("no score bounds recorded for this update")
        mx = float(self.maximum)
        if not math.isfinite(mx) or mx < 0:
            raise FloatingPointError("nonfinite or negative score bound; update aborted")
        return mx

    def clip(self, tau):
        from .qk_clip import qk_clip_from_bounds_
        self.finish_update()
        if self.last is None:
            raise ValueError("no last-microbatch score bounds for clipping")
        for blk, bounds in zip(self.model.blocks, self.last):
            blk.attn.last_score_bound = bounds
        t0 = time.monotonic()
        stats = qk_clip_from_bounds_(self.model, tau)
        bad = []
        finite_json(stats, "qk_clip", bad)
        if bad:
            raise FloatingPointError("nonfinite QK clipping result: " + ", ".join(bad))
        return {**stats, "seconds": time.monotonic() - t0, "optimizer_state_policy": "moments and step counters unchanged"}


class TrainingStabilityProbe:
    """First row (<= 512 tokens) of an independent train-split sampler, used between optimizer
    steps for stability statistics and probe-based QK-clip; RNG, module modes and norm collection
    state are restored afterwards."""

    def __init__(self, cfg, device):
        from .data import PackedSampler, batch_hash
        self.device = torch.device(device)
        data = cfg.raw["data"]
        context = min(data.get("context", 512), 512)
        sampler = PackedSampler(data["manifest"], split="train", batch_size=1, context=context, seed=cfg.train.seed)
        batch = sampler.next_batch()
        self.identity = {"batch_sha256": batch_hash(batch), "manifest_sha256": sampler.manifest_hash, "split": "train",
                         "seed": cfg.train.seed, "context": context, "batch_size": 1}
        self.idx, self.doc = (t.to(self.device) for t in batch[:2])

    def _run(self, model, operation):
        t0 = time.monotonic()
        modes = [(m, m.training) for m in model.modules()]
        norms = [(m, m.collecting, m._valid) for m in lagged_modules(model) + taper_modules(model)]
        bounds = [(b.attn, b.attn.record_score_bound, b.attn.last_score_bound) for b in model.blocks]
        py_rng, np_rng = random.getstate(), np.random.get_state()
        devices = ([self.device.index if self.device.index is not None else torch.cuda.current_device()]
                   if self.device.type == "cuda" else [])
        try:
            with torch.random.fork_rng(devices=devices), torch.no_grad():
                model.eval()
                for attn, _, _ in bounds:
                    attn.record_score_bound = False
                for m, _, _ in norms:
                    m.collecting = False
                stats = operation(model, self.idx, self.doc)
                if self.device.type == "cuda":
                    torch.cuda.synchronize(self.device)
        finally:
            for attn, rec, last in bounds:
                attn.record_score_bound, attn.last_score_bound = rec, last
            for m, training in modes:
                m.training = training
            for m, coll, valid in norms:
                m.collecting, m._valid = coll, valid
            random.setstate(py_rng)
            np.random.set_state(np_rng)
        return stats, time.monotonic() - t0

    def sample(self, model) -> dict:
        from .analysis import stability_stats
        stats, seconds = self._run(model, stability_stats)
        bad = []
        clean = finite_json(stats, "stats", bad)
        return {"stats": clean, "probe": dict(self.identity), "seconds": seconds, "nonfinite_paths": bad}

    def clip(self, model, tau) -> dict:
        from .qk_clip import qk_clip_
        stats, seconds = self._run(model, lambda m, idx, doc: qk_clip_(m, idx, doc, tau))
        bad = []
        finite_json(stats, "qk_clip", bad)
        if bad:
            raise FloatingPointError("nonfinite QK clipping result: " + ", ".join(bad))
        return {**stats, "probe": dict(self.identity), "seconds": seconds,
                "optimizer_state_policy": "moments and step counters unchanged"}
