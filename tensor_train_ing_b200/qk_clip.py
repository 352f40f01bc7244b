"""QK-clip for polynomial attention: after an update, rescale each head whose max |S| exceeds tau
by sqrt(tau / max) on its Q and K rows, so that head's max |S| becomes tau exactly, per factor
(S1 from q1/k1, S2 from q2/k2).  Probe-based (exact on the probe, sequential over layers with
re-measurement) or from the per-batch Cauchy-Schwarz bounds recorded during the training forward
(conservative, layers independent).  Reference: tnlm/qk_clip.py:21-96."""
from __future__ import annotations

import torch

from .models.normalization import SpectralLinear


@torch.no_grad()
def head_score_max(model, idx, doc) -> list[dict]:
    """Per layer {'S1': (H,), 'S2': (H,)}: max |S| over visible pairs of the probe's first row."""
    from .analysis import probe_attention_scores
    scores, _, vis = probe_attention_scores(model, idx, doc, max_tokens=idx.shape[1])
    return [{k: S.masked_fill(~vis, 0).abs().amax(dim=(-1, -2)) for k, S in row.items()} for row in scores]


@torch.no_grad()
def _rescale_heads_(blk, name: str, gamma: torch.Tensor, d_key: int):
    q, k = (blk.attn.q1, blk.attn.k1) if name == "S1" else (blk.attn.q2, blk.attn.k2)
    rows = gamma.sqrt().repeat_interleave(d_key).to(q.weight.dtype)
    for lin in (q, k):
        if not getattr(lin.weight, "_ttb_remote", False):  # sharded: only the owner holds the master
            lin.weight.mul_(rows[:, None])
        if lin.bias is not None:
            lin.bias.mul_(rows)


def _no_spectral(model):
    if any(isinstance(m, SpectralLinear) for m in model.modules()):
        raise NotImplementedError("QK-clip is exact only for plain linear Q/K (not spectral_rms)")


@torch.no_grad()
def qk_clip_(model, idx, doc, tau: float) -> dict:
    if tau <= 0:
        raise ValueError("tau must be positive")
    _no_spectral(model)
    clipped, worst, factors = 0, 0.0, {}
    for i, blk in enumerate(model.blocks):
        stats = head_score_max(model, idx, doc)[i]  # re-measured after the earlier layers were clipped
        for name, mx in stats.items():
            worst = max(worst, float(mx.max()))
            gamma = torch.clamp(tau / mx.clamp_min(1e-30), max=1.0)
            if bool((gamma < 1).any()):
                _rescale_heads_(blk, name, gamma, model.cfg.d_key)
                clipped += int((gamma < 1).sum())
                factors.setdefault(i, {})[name] = [float(g) for g in gamma]
    return {"clipped_heads": clipped, "max_before": worst, "factors": factors, "tau": tau}


def set_score_bound_recording(model, on: bool = True):
    for blk in model.blocks:
        blk.attn.record_score_bound = on
        if not on:
            blk.attn.last_score_bound = None


def score_bounds(model) -> list[dict]:
    return [dict(blk.attn.last_score_bound or {}) for blk in model.blocks]


@torch.no_grad()
def qk_clip_from_bounds_(model, tau: float) -> dict:
    if tau <= 0:
        raise ValueError("tau must be positive")
    _no_spectral(model)
    clipped, worst, factors = 0, 0.0, {}
    for i, (blk, stats) in enumerate(zip(model.blocks, score_bounds(model))):
        for name, bound in stats.items():
            worst = max(worst, float(bound.max()))
            gamma = torch.clamp(tau / bound.clamp_min(1e-30), max=1.0)
            if bool((gamma < 1).any()):
                _rescale_heads_(blk, name, gamma, model.cfg.d_key)
                clipped += int((gamma < 1).sum())
                factors.setdefault(i, {})[name] = [float(g) for g in gamma]
    return {"clipped_heads": clipped, "max_bound_before": worst, "factors": factors, "tau": tau,
            "source": "per-batch norm bound"}
