"""Fused (sm_100a) execution of ``TensorLM``: context tables, block forward and model forward.

Per block (reference tnlm/model.py:137-144, 67-101):
  h   = norm_in(x)                       RMSNorm / GroupRMSNorm / lagged / taper kernel -> bf16
  qkv = h [q1|k1|q2|k2|v]^T              one tcgen05 GEMM over the concatenated bf16 weights, RoPE in place
  y   = PolyAttention(qkv)               tcgen05 attention kernels
  x   = x + alpha * o(y)                 GEMM with the residual add in its epilogue (fp32 stream)
  x   = x + alpha * D(L h' * R h')       dual-B bilinear GEMM, then the down GEMM with fused residual
With an output norm (branch_rms / sandwich_rms) the bf16 branch output goes through one kernel that
forms x + alpha * RMSNorm(branch) in fp32.  Spectral layers feed the GEMMs bf16(gamma W / sigma) from one
kernel pass per layer and turn dW_eff into dW and dgamma with another.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..models.attention import rope_inv_freq, row_scale_vector
from ..models.normalization import GroupRMSNorm, LaggedRMS, RMSNorm, SpectralLinear, TaperRMS
from . import fused, norms
from .weights import group_for, spectral_group_for


def _weights(owner, name, linears):
    if any(isinstance(l, SpectralLinear) for l in linears):
        if not all(isinstance(l, SpectralLinear) and l.weight.shape[1] % 4 == 0 for l in linears):
            raise ValueError("a fused weight group mixes spectral and plain layers")
        return spectral_group_for(owner, name, linears)
    return group_for(owner, name, [l.weight for l in linears])


def model_weight_groups(model):
    """Every (owner, name, linears) weight group the fused path uses, in backward order
    (unembed first, then blocks from last to first, embedding last).  Spectral layers are
    excluded (their effective weights are recomputed every forward)."""
    out = [(model, "unembed", [model.unembed])]
    for blk in reversed(model.blocks):
        a, m = blk.attn, blk.mlp
        for owner, name, lins in ((m, "d", [m.d]), (m, "r", [m.r]), (m, "l", [m.l]), (a, "o", [a.o]),
                                  (a, "qkv", a.projections())):
            if not any(isinstance(l, SpectralLinear) for l in lins):
                out.append((owner, name, lins))
    out.append((model, "embed", [model.embed]))
    return out


def rope_context(pos32: torch.Tensor, T: int, dk: int, base: float) -> dict:
    """cos/sin tables [T, dk/2] computed exactly as the reference's rope_tables (fp32 torch ops),
    indexed by position-in-document inside the kernels."""
    positions = torch.arange(T, device=pos32.device)
    angle = positions.float().unsqueeze(-1) * rope_inv_freq(dk, base, pos32.device)
    return {"pos32": pos32, "cos": angle.cos().contiguous(), "sin": angle.sin().contiguous()}


def fused_context(model, doc_ids, pos):
    cfg = model.cfg
    tables = fused.attention_tables(doc_ids)
    row_scale = {p: row_scale_vector(doc_ids, p).contiguous().view(-1) for p in model._row_powers()}
    rope = rope_context(tables["pos32"], tables["T"], cfg.d_key, cfg.rope_base)
    return {"fused": True, "tables": tables, "row_scale": row_scale, "rope": rope}


def norm_to_bf16(norm: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """Apply an input norm to the fp32 stream and return the bf16 GEMM operand."""
    if isinstance(norm, nn.Identity):
        return x.to(torch.bfloat16)
    if isinstance(norm, (RMSNorm, GroupRMSNorm)) and norm.denom_mode is None:
        groups = norm.groups if isinstance(norm, GroupRMSNorm) else 1
        return fused.rms_norm(x, norm.weight, groups, norm.eps)
    if isinstance(norm, LaggedRMS) and x.shape[-1] % 4 == 0:
        return norms.lagged_to_bf16(norm, x)
    if isinstance(norm, TaperRMS) and x.shape[-1] % 4 == 0:
        return norms.taper_to_bf16(norm, x)
    return norm(x).to(torch.bfloat16)


def _add_branch(x, out_norm, branch, alpha):
    """x + alpha * out_norm(branch) for a branch-output norm (fp32 stream)."""
    if type(out_norm) is RMSNorm and out_norm.denom_mode is None and branch.shape[-1] % 4 == 0:
        return norms.output_rms(x, branch.float(), out_norm, alpha)
    return x + alpha * out_norm(branch)


def _record_bound(attn, norms):
    """Per head max |q| max |k| / sqrt(dk) from the per-head maximum row norms the QKV epilogue
    wrote (rotated heads in buffer order: q1, k1[, q2, k2])."""
    H, dk = attn.cfg.heads, attn.cfg.d_key
    per = norms.view(-1, H)
    bounds = {"S1": per[0] * per[1] / dk ** 0.5}
    if attn.kind != "offset_square":
        bounds["S2"] = per[2] * per[3] / dk ** 0.5
    attn.last_score_bound = bounds


def attention_branch(blk, h, ctx):
    a = blk.attn
    cfg = a.cfg
    H, dk, dv = cfg.heads, cfg.d_key, cfg.d_value
    projs = a.projections()
    grp = _weights(a, "qkv", projs)
    two = a.kind != "offset_square"
    n_qk = 4 if two else 2
    norms = torch.zeros(n_qk * H, device=h.device, dtype=torch.float32) if a.record_score_bound else None
    qkv = fused.qkv_rope(h, grp, n_qk * H * dk, dk, ctx["rope"], norms)
    if two:
        cols = [0, H * dk, 2 * H * dk, 3 * H * dk, 4 * H * dk]
    else:
        cols = [0, H * dk, 0, H * dk, 2 * H * dk]
    if norms is not None:
        _record_bound(a, norms)
    kpar = getattr(a, "b", None) if a.kind == "offset_square" else getattr(a, "coef", None)
    return fused.poly_attention(qkv, kpar, a.kind, dk, dv, H, cols, ctx["tables"], ctx["row_scale"][a.row_power],
                                ctx["rope"])


def _split_norm(norm) -> bool:
    return isinstance(norm, (RMSNorm, GroupRMSNorm)) and norm.denom_mode is None


def _norm_and_residual(norm, x, up_alpha):
    """(residual stream, bf16 branch input).  Plain RMS / group norms go through ResidualNormFn,
    whose backward folds the norm's dx into the residual gradient in place and emits the bf16
    operand of the upstream branch's backward GEMM (``up_alpha`` = that branch's alpha, None when
    the stream was not produced by a fused residual GEMM)."""
    if _split_norm(norm):
        groups = norm.groups if isinstance(norm, GroupRMSNorm) else 1
        return fused.residual_norm(x, norm.weight, groups, norm.eps, up_alpha)
    return x, norm_to_bf16(norm, x)


def _fused_residual(blk, branch):
    return branch not in blk.ablate and isinstance(getattr(blk, f"{branch}_out"), nn.Identity)


def _output_alpha(blk, incoming):
    """Alpha of the fused residual GEMM that produced the block's output stream (None if not fused)."""
    if "mlp" not in blk.ablate:
        return blk.alpha if _fused_residual(blk, "mlp") else None
    if "attn" not in blk.ablate:
        return blk.alpha if _fused_residual(blk, "attn") else None
    return incoming


def block_forward(blk, x, ctx):
    """x: fp32 [N, d] residual stream."""
    a, m = blk.attn, blk.mlp
    up = getattr(blk, "_ttb_up_alpha", None)  # set per block by model_forward (structure only)
    if "attn" not in blk.ablate:
        x, h = _norm_and_residual(blk.attn_in, x, up)
        y = attention_branch(blk, h, ctx)
        og = _weights(a, "o", [a.o])
        if isinstance(blk.attn_out, nn.Identity):
            x = fused.linear(y, og, residual=x, alpha=blk.alpha, bias=a.o.bias)
            up = blk.alpha
        else:
            x = _add_branch(x, blk.attn_out, fused.linear(y, og, bias=a.o.bias), blk.alpha)
            up = None
    if "mlp" not in blk.ablate:
        x, h = _norm_and_residual(blk.mlp_in, x, up)
        gl, gr, gd = _weights(m, "l", [m.l]), _weights(m, "r", [m.r]), _weights(m, "d", [m.d])
        mode = 1 if m.kind == "swiglu" else 0
        if isinstance(blk.mlp_out, nn.Identity):
            x = fused.bilinear_mlp(h, gl, gr, gd, residual=x, alpha=blk.alpha, mode=mode,
                                   bl=m.l.bias, br=m.r.bias, bd=m.d.bias)
        else:
            branch = fused.bilinear_mlp(h, gl, gr, gd, mode=mode, bl=m.l.bias, br=m.r.bias, bd=m.d.bias)
            x = _add_branch(x, blk.mlp_out, branch, blk.alpha)
    return x


def model_forward(model, idx, ctx, targets, reduction):
    cfg = model.cfg
    B, T = idx.shape
    x = fused.embedding(idx.reshape(-1), group_for(model, "embed", [model.embed.weight]))
    up = None  # the embedding's backward takes the fp32 gradient directly
    for blk in model.blocks:
        object.__setattr__(blk, "_ttb_up_alpha", up)
        up = _output_alpha(blk, up)
    recompute = model.recomputed_blocks()
    for i, blk in enumerate(model.blocks):
        if i < recompute:
            x = torch.utils.checkpoint.checkpoint(block_forward, blk, x, ctx, use_reentrant=False)
        else:
            x = blk(x, ctx)
    h = norm_to_bf16(model.final_norm, x)
    V = cfg.vocab_size
    ug = group_for(model, "unembed", [model.unembed.weight])
    alpha = model.logit_multiplier
    if targets is not None and cfg.loss_chunk_tokens > 0:
        loss = fused.linear_cross_entropy(h, targets.reshape(-1), ug, V, alpha, cfg.loss_chunk_tokens)
        logits = None
    else:
        logits = fused.linear(h, ug)[:, :V].view(B, T, V)
        if alpha != 1.0:
            logits = logits * alpha
        if targets is None:
            return logits
        loss = torch.nn.functional.cross_entropy(logits.float().flatten(0, 1), targets.flatten(),
                                                 ignore_index=-100, reduction="sum")
    n = (targets != -100).sum()
    if reduction == "sum":
        return logits, loss, n
    return logits, loss / n.clamp_min(1)
