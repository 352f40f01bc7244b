"""Chunked linear + cross-entropy in plain PyTorch (the reference/CPU path).

Exact, with bounded logit memory: the forward keeps only the per-token log-sum-exp and the
backward recomputes each chunk's logits (reference tnlm/kernels/fused_ce.py:18-60).  On CUDA the
model uses ``ops.fused.linear_cross_entropy`` (logits never stored in the forward).
"""
from __future__ import annotations

import torch


def _compute_dtype(x):
    if torch.is_autocast_enabled(x.device.type):
        return torch.get_autocast_dtype(x.device.type)
    return x.dtype


class ChunkedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, targets, chunk, cdtype):
        acc_dtype = torch.promote_types(cdtype, torch.float32)
        xc, wc = x.to(cdtype), w.to(cdtype)
        valid = targets != -100
        safe = targets.clamp_min(0)
        lse = torch.empty(x.shape[0], device=x.device, dtype=acc_dtype)
        total = torch.zeros((), device=x.device, dtype=acc_dtype)
        for s in range(0, x.shape[0], chunk):
            logits = (xc[s:s + chunk] @ wc.t()).to(acc_dtype)
            l = torch.logsumexp(logits, dim=-1)
            lse[s:s + chunk] = l
            picked = logits.gather(1, safe[s:s + chunk, None]).squeeze(1)
            total += ((l - picked) * valid[s:s + chunk]).sum()
        ctx.save_for_backward(x, w, targets, lse)
        ctx.chunk, ctx.cdtype = chunk, cdtype
        return total

    @staticmethod
    def backward(ctx, g):
        x, w, targets, lse = ctx.saved_tensors
        xc, wc = x.to(ctx.cdtype), w.to(ctx.cdtype)
        valid = targets != -100
        safe = targets.clamp_min(0)
        dx = torch.empty_like(x)
        dw = torch.zeros(w.shape, device=w.device, dtype=lse.dtype)
        for s in range(0, x.shape[0], ctx.chunk):
            sl = slice(s, s + ctx.chunk)
            p = torch.exp((xc[sl] @ wc.t()).to(lse.dtype) - lse[sl, None])
            p.scatter_add_(1, safe[sl, None], -torch.ones_like(p[:, :1]))
            p = (p * (valid[sl, None] * g)).to(ctx.cdtype)
            dx[sl] = (p @ wc).to(x.dtype)
            dw += (p.t() @ xc[sl]).to(lse.dtype)
        return dx, dw.to(w.dtype), None, None, None


def chunked_linear_cross_entropy_reference(x, w, targets, chunk=4096):
    """Sum over valid targets of CE(x @ w.T, target); x: (N, d), w: (V, d), targets: (N,)."""
    return ChunkedLinearCE.apply(x, w, targets, chunk, _compute_dtype(x))


linear_cross_entropy_sum = chunked_linear_cross_entropy_reference
