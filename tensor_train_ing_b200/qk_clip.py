"""QK-clip for polynomial attention: bound each head's attention scores by rescaling its weights.

After an optimizer update, a head whose largest |S| = |q.k| / sqrt(dk) exceeds ``tau`` gets its query
and key rows multiplied by sqrt(tau / max), which multiplies its scores by exactly tau / max; S1 (from
q1, k1) and S2 (from q2, k2) are clipped separately, so S1*S2 stays within tau**2.  Only weights
change (no optimizer state), so the model stays exactly polynomial and exports stay linear maps.
Two sources for the maxima, as in the reference (tnlm/qk_clip.py:21-96):

* ``qk_clip_``: a fixed probe row, layer after layer, re-measured after each clipped layer (clipping
  layer i changes what layer i+1 reads); exact on the probe, not a bound on unseen data;
* ``qk_clip_from_bounds_``: the per-head Cauchy-Schwarz bounds max|q|*max|k|/sqrt(dk) the last
  training forward recorded; every score of that batch ends at or below tau (it may over-clip), and
  the layers are independent.

A spectrally reparametrised Q/K (W/sigma(W)) would change sigma under a row rescale, so the clip
would not be exact; such models are refused.
"""
from __future__ import annotations

import torch

from .models.normalization import SpectralLinear

FACTOR_WEIGHTS = {"S1": ("q1", "k1"), "S2": ("q2", "k2")}


def set_score_bound_recording(model, on: bool = True) -> None:
    for blk in model.blocks:
        blk.attn.record_score_bound = on
        if not on:
            blk.attn.last_score_bound = None


def score_bounds(model) -> list[dict]:
    """Per layer, the {factor: (H,) bound} of the last forward that recorded them ({} if none)."""
    return [dict(blk.attn.last_score_bound or {}) for blk in model.blocks]


@torch.no_grad()
def head_score_max(model, idx, doc) -> list[dict]:
    """Per layer, {factor: (H,)} largest |S| over causally visible same-document pairs of the probe."""
    from .analysis import probe_attention_scores
    scores, _, visible = probe_attention_scores(model, idx, doc, max_tokens=idx.shape[1])
    return [{f: s.masked_fill(~visible, 0).abs().amax(dim=(-1, -2)) for f, s in layer.items()} for layer in scores]


@torch.no_grad()
def scale_head_rows(block, factor: str, per_head: torch.Tensor, d_key: int) -> None:
    """Multiply each head's rows of the factor's Q and K projections by ``per_head[h]``."""
    rows = per_head.repeat_interleave(d_key)
    for name in FACTOR_WEIGHTS[factor]:
        lin = getattr(block.attn, name)
        # a parameter-sharded non-owner holds no master: its owner scales and the gather brings it
        if not getattr(lin.weight, "_ttb_remote", False):
            lin.weight.mul_(rows.to(lin.weight.dtype)[:, None])
        if lin.bias is not None:
            lin.bias.mul_(rows.to(lin.bias.dtype))


class _Tally:
    def __init__(self, tau: float):
        self.tau = tau
        self.heads = 0
        self.worst = 0.0
        self.factors: dict = {}

    def clip(self, layer: int, block, factor: str, maxima: torch.Tensor, d_key: int) -> None:
        self.worst = max(self.worst, float(maxima.max()))
        gamma = (self.tau / maxima.clamp_min(1e-30)).clamp(max=1.0)
        over = gamma < 1
        if bool(over.any()):
            scale_head_rows(block, factor, gamma.sqrt(), d_key)
            self.heads += int(over.sum())
            self.factors.setdefault(layer, {})[factor] = gamma.tolist()


def _start(model, tau: float) -> _Tally:
    if not tau > 0:
        raise ValueError("the QK-clip threshold tau must be positive")
    if any(isinstance(m, SpectralLinear) for m in model.modules()):
        raise NotImplementedError("QK-clip is exact only for plain linear Q/K projections (not spectral_rms)")
    return _Tally(float(tau))


@torch.no_grad()
def qk_clip_(model, idx, doc, tau: float) -> dict:
    tally = _start(model, tau)
    for layer, blk in enumerate(model.blocks):
        for factor, maxima in head_score_max(model, idx, doc)[layer].items():
            tally.clip(layer, blk, factor, maxima, model.cfg.d_key)
    return {"clipped_heads": tally.heads, "max_before": tally.worst, "factors": tally.factors, "tau": tau}


@torch.no_grad()
def qk_clip_from_bounds_(model, tau: float) -> dict:
    tally = _start(model, tau)
    for layer, (blk, bounds) in enumerate(zip(model.blocks, score_bounds(model))):
        for factor, bound in bounds.items():
            tally.clip(layer, blk, factor, bound, model.cfg.d_key)
    return {"clipped_heads": tally.heads, "max_bound_before": tally.worst, "factors": tally.factors, "tau": tau,
            "source": "per-batch norm bound"}
