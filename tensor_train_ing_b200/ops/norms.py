"""Fused-path forms of the normalisation variants: lagged RMS, TaperNorm and the fp32-output RMSNorm
that ``branch_rms`` / ``sandwich_rms`` apply to branch outputs (csrc/misc/norm_variants.cu).

Each returns what the fused block needs (the bf16 GEMM operand for input norms, the updated fp32
residual stream for output norms) and keeps the modules' training-time bookkeeping: lagged
statistics collection, TaperNorm warm-up statistics and the differentiable anchor term (the kernel
returns the per-row r, whose gradient the backward kernel folds into dx).  The module forwards in
models/normalization.py remain the definition these are tested against.
"""
from __future__ import annotations

import torch

from ._ext import lib

LAGGED, TAPER, RMS = 0, 1, 2


class LaggedNormFn(torch.autograd.Function):
    """bf16(x * s * w) with s = 1 / sqrt(mean_sq + eps), a detached device scalar."""

    @staticmethod
    def forward(ctx, x, w, scale, eps, want_msq):
        y16, _, _, msq = lib().norm_variant_fwd(x, w, None, LAGGED, 0.0, 0.0, scale, eps, True, False, None, 1.0,
                                                False, bool(want_msq))
        if msq is None:
            msq = x.new_empty(0)
        ctx.save_for_backward(x, w, scale)
        ctx.eps = eps
        ctx.mark_non_differentiable(msq)
        return y16, msq

    @staticmethod
    def backward(ctx, dy, _dmsq):
        x, w, scale = ctx.saved_tensors
        dx, dw, _ = lib().norm_variant_bwd(dy.contiguous(), x, w, None, LAGGED, 0.0, 0.0, scale, ctx.eps, 1.0, None,
                                           None, None, False, ctx.needs_input_grad[1], False)
        return dx, (dw if ctx.needs_input_grad[1] else None), None, None, None


class TaperNormFn(torch.autograd.Function):
    """(bf16(x * (g/r * w + b * w2)), r) with b = (1 - g) c and r = sqrt(mean x^2 + eps) per row."""

    @staticmethod
    def forward(ctx, x, w, w2, g, b, eps):
        y16, _, r, _ = lib().norm_variant_fwd(x, w, w2, TAPER, g, b, None, eps, True, False, None, 1.0, True, False)
        ctx.save_for_backward(x, w, w2, r)
        ctx.g, ctx.b, ctx.eps = g, b, eps
        return y16, r

    @staticmethod
    def backward(ctx, dy, dr):
        x, w, w2, r = ctx.saved_tensors
        want_w = ctx.needs_input_grad[1] and ctx.g != 0.0
        want_w2 = ctx.needs_input_grad[2] and ctx.b != 0.0
        dx, dw, dw2 = lib().norm_variant_bwd(dy.contiguous(), x, w, w2 if ctx.b != 0.0 else None, TAPER, ctx.g,
                                             ctx.b, None, ctx.eps, 1.0, r,
                                             dr.contiguous() if dr is not None else None, None, False, want_w,
                                             want_w2)
        return dx, (dw if want_w else None), (dw2 if want_w2 else None), None, None, None


class OutputRmsFn(torch.autograd.Function):
    """resid + alpha * rmsnorm(z) * w in fp32 (one pass; the branch output never becomes an extra
    tensor)."""

    @staticmethod
    def forward(ctx, resid, z, w, alpha, eps):
        _, y32, r, _ = lib().norm_variant_fwd(z, w, None, RMS, 0.0, 0.0, None, eps, False, True, resid, alpha, True,
                                              False)
        ctx.save_for_backward(z, w, r)
        ctx.alpha, ctx.eps = alpha, eps
        return y32

    @staticmethod
    def backward(ctx, dy):
        z, w, r = ctx.saved_tensors
        dy = dy.contiguous()
        dz, dw, _ = lib().norm_variant_bwd(dy, z, w, None, RMS, 0.0, 0.0, None, ctx.eps, ctx.alpha, r, None, None,
                                           False, ctx.needs_input_grad[2], False)
        return dy, dz, (dw if ctx.needs_input_grad[2] else None), None, None


def _valid_rows(norm, n_rows):
    valid = getattr(norm, "_valid", None)
    return None if valid is None else valid.reshape(-1)[:n_rows].double()


def lagged_to_bf16(norm, x):
    """LaggedRMS on the fused path: the bf16 operand, and (while collecting) the per-token mean squares
    folded into the module's count-weighted sums, padding excluded."""
    scale = (norm.mean_sq + norm.eps).sqrt().reciprocal().to(torch.float32).reshape(1)
    y16, msq = LaggedNormFn.apply(x, norm.weight, scale, float(norm.eps), norm.collecting)
    if norm.collecting:
        with torch.no_grad():
            per_row = msq.double()
            valid = _valid_rows(norm, x.shape[0])
            if valid is not None:
                norm.acc_sum += (per_row * valid).sum()
                norm.acc_count += valid.sum()
            else:
                norm.acc_sum += per_row.sum()
                norm.acc_count += float(per_row.numel())
    return y16


def taper_to_bf16(norm, x):
    """TaperRMS on the fused path, with its warm-up statistics and anchor accumulation."""
    g = float(norm.gate)
    frozen = bool(norm.frozen)
    b = (1.0 - g) * float(norm.c)
    y16, r = TaperNormFn.apply(x, norm.weight, norm.weight_tilde, g, b, float(norm.eps))
    valid = _valid_rows(norm, x.shape[0])
    if norm.collecting and not frozen:
        with torch.no_grad():
            sq = (x.detach() * norm.weight.detach()).double().square().sum(dim=-1)
            rr = r.detach().double()
            wv = valid if valid is not None else torch.ones_like(rr)
            norm.acc_num += (sq / rr * wv).sum()
            norm.acc_den += (sq * wv).sum()
            norm.acc_r += (rr * wv).sum()
            norm.acc_count += wv.sum()
    if norm.training and frozen:
        dev = (r - norm.s_tgt.to(r.dtype)).square()
        if valid is not None:
            dev = dev * valid.to(dev.dtype)
            count = float(valid.sum())
        else:
            count = float(dev.numel())
        total = dev.sum()
        norm._anchor_sum = total if norm._anchor_sum is None else norm._anchor_sum + total
        norm._anchor_count += count
    return y16


def output_rms(resid, z, norm, alpha):
    """``resid + alpha * norm(z)`` for an RMSNorm applied to a branch output (fp32 stream)."""
    return OutputRmsFn.apply(resid.contiguous(), z.contiguous(), norm.weight, float(alpha), float(norm.eps))
