"""Autograd functions over the sm_100a kernels (tcgen05 GEMMs, polynomial attention, norms,
fused linear-CE, embedding).  Every function here runs only on the compiled library; there is
no PyTorch fallback inside (see ``ops._ext``).

Conventions: the residual stream is fp32 [N, d]; GEMM operands are bf16; weight gradients are
accumulated through ``WeightGroup.sink_grad`` (fp32, in the GEMM epilogue).
"""
from __future__ import annotations

import contextlib

import torch

from ._ext import lib


# (M, N, K) -> output tile width (128 or 256) chosen by ``tensor_train_ing_b200.tune``; absent shapes
# take the kernel's own choice (128 for N <= 128, else the 256-wide CTA-pair tile)
GEMM_TILES: dict[tuple[int, int, int], int] = {}


def _mm(a, b, out, c=None, alpha=1.0, beta=0.0, bias=None, b2=None, gather=None):
    """out = alpha * (a @ b + bias) + beta * c; with ``b2``, a @ cat(b, b2) in one pass.  ``gather``:
    b is the transpose of a staging buffer that the GEMM fills from the ranks' row shards first."""
    tile = GEMM_TILES.get((out.shape[0], out.shape[1], a.shape[1]), 0) if GEMM_TILES else 0
    lib().mm(a, b, out, c, float(alpha), float(beta), bias, b2, tile, gather)
    return out


def _gathers(*specs):
    """Gather descriptions of a GEMM's staged operands, as the kernels take them (None: nothing to
    gather)."""
    return [s for s in specs] if all(s is not None for s in specs) else None


@contextlib.contextmanager
def _launching(*pairs):
    """Around a launch that gathers its weights: when the launch is refused on the host, the groups'
    window slots and done words are put back so the next request gathers from scratch."""
    try:
        yield
    except Exception:
        for group, spec in pairs:
            gw = getattr(group, "_gather", None)
            if spec is not None and gw is not None:
                gw.window.release(gw)
                gw.reset()
        raise


# ============================================================================ RMSNorm
class RMSNormFn(torch.autograd.Function):
    """y = bf16(x / rms_g(x) * w) for fp32 x [N, d]; groups > 1 = GroupRMSNorm."""

    @staticmethod
    def forward(ctx, x, w, groups, eps):
        y, rstd = lib().rmsnorm_fwd(x, w, int(groups), float(eps))
        ctx.save_for_backward(x, w, rstd)
        ctx.groups = int(groups)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx = torch.empty_like(x)
        dw = lib().rmsnorm_bwd(dy.contiguous(), x, w, rstd, dx, False, ctx.groups)
        return dx, dw, None, None


def rms_norm(x, w, groups=1, eps=1e-6):
    return RMSNormFn.apply(x.contiguous(), w.contiguous(), groups, eps)


def _take_bf16(dout, alpha):
    """The bf16 operand bf16(alpha * dout) for a backward GEMM: the copy the residual-norm backward
    attached to ``dout`` when it matches, else a conversion."""
    pre = getattr(dout, "_ttb_bf16", None)
    if pre is not None and pre[1] == alpha and pre[0].shape == dout.shape:
        return pre[0]
    if alpha != 1.0 or dout.dtype != torch.bfloat16:
        return (dout * alpha).to(torch.bfloat16).contiguous()
    return dout.contiguous()


class ResidualNormFn(torch.autograd.Function):
    """(x, h): x passes through to the residual add, h = bf16(x / rms_g(x) * w) feeds the branch.

    Backward: the fp32 residual gradient is updated in place with the norm's dx by the RMSNorm
    backward kernel, which in the same pass writes bf16(up_alpha * dx_total), the operand the
    producing branch's backward GEMM needs (attached to the gradient tensor)."""

    @staticmethod
    def forward(ctx, x, w, groups, eps, up_alpha):
        h, rstd = lib().rmsnorm_fwd(x, w, int(groups), float(eps))
        ctx.save_for_backward(x, w, rstd)
        ctx.groups, ctx.up_alpha = int(groups), up_alpha
        return x.view_as(x), h

    @staticmethod
    def backward(ctx, dres, dh):
        x, w, rstd = ctx.saved_tensors
        accumulate = dres is not None
        if not accumulate or dres.dtype != torch.float32 or not dres.is_contiguous():
            dres = torch.empty_like(x) if not accumulate else dres.float().contiguous().clone()
        if dh is None:
            dh = torch.zeros(x.shape, device=x.device, dtype=torch.bfloat16)
        g16 = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16) if ctx.up_alpha is not None else None
        dw = lib().rmsnorm_bwd(dh.contiguous(), x, w, rstd, dres, accumulate, ctx.groups, g16,
                               float(ctx.up_alpha) if ctx.up_alpha is not None else 1.0)
        if g16 is not None:
            dres._ttb_bf16 = (g16, ctx.up_alpha)
        elif hasattr(dres, "_ttb_bf16"):
            del dres._ttb_bf16
        return dres, dw, None, None, None


def residual_norm(x, w, groups=1, eps=1e-6, up_alpha=None):
    return ResidualNormFn.apply(x.contiguous(), w.contiguous(), groups, eps, up_alpha)


# ============================================================================ linear
class LinearFn(torch.autograd.Function):
    """out = residual + alpha * (x W^T + b)  (fp32, residual given)  or  bf16(x W^T + b).

    x: bf16 [N, d_in]; ``group`` provides the bf16 weight and the gradient sink."""

    @staticmethod
    def forward(ctx, x, residual, bias, group, alpha, *weights):
        w16, spec = group.operand()
        N = x.shape[0]
        with _launching((group, spec)):
            if residual is not None:
                out = torch.empty(N, w16.shape[0], device=x.device, dtype=torch.float32)
                _mm(x, w16.t(), out, c=residual, alpha=alpha, beta=1.0, bias=bias, gather=_gathers(spec))
            else:
                out = torch.empty(N, w16.shape[0], device=x.device, dtype=torch.bfloat16)
                _mm(x, w16.t(), out, alpha=alpha, bias=bias, gather=_gathers(spec))
        ctx.save_for_backward(x)
        ctx.group, ctx.alpha, ctx.has_res, ctx.has_bias = group, alpha, residual is not None, bias is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        (x,) = ctx.saved_tensors
        group, alpha = ctx.group, ctx.alpha
        # gradient of the branch output, as the bf16 operand of the backward GEMMs
        g = _take_bf16(dout, alpha)
        w16 = group.bf16()
        dx = torch.empty_like(x)
        _mm(g, w16, dx)
        grads = group.sink_grad(lambda out, beta: _mm(g.t(), x, out, c=out, beta=beta))
        dres = dout if ctx.has_res else None
        dbias = g.float().sum(0) if ctx.has_bias else None
        return (dx, dres, dbias, None, None, *grads)


def linear(x, group, residual=None, alpha=1.0, bias=None):
    return LinearFn.apply(x, residual, bias, group, float(alpha), *group.params)


# ============================================================================ QKV + RoPE
class QKVRopeFn(torch.autograd.Function):
    """qkv = x W_cat^T (bf16 [N, sum rows]) with RoPE on the first rope_cols columns, applied in the
    GEMM epilogue.  The backward receives a gradient that the attention backward has already
    rotated back (it writes dq/dk w.r.t. the pre-rotation projections), so only GEMMs remain."""

    @staticmethod
    def forward(ctx, x, group, rope_cols, dk, rope, norm_max, *weights):
        w16, spec = group.operand()
        with _launching((group, spec)):
            qkv = lib().qkv_rope(x, w16, int(rope_cols), int(dk), rope["pos32"], rope["cos"], rope["sin"], norm_max,
                                 _gathers(spec))
        ctx.save_for_backward(x)
        ctx.group = group
        return qkv

    @staticmethod
    def backward(ctx, dqkv):
        (x,) = ctx.saved_tensors
        if not getattr(dqkv, "_ttb_unrotated", False):
            raise RuntimeError("QKVRopeFn expects the gradient produced by PolyAttentionFn (rotary already undone)")
        g = dqkv.contiguous()
        w16 = ctx.group.bf16()
        dx = torch.empty_like(x)  # bf16 like the input: no cast inserted by autograd
        _mm(g, w16, dx)
        grads = ctx.group.sink_grad(lambda out, beta: _mm(g.t(), x, out, c=out, beta=beta))
        return (dx, None, None, None, None, None, *grads)


def qkv_rope(x, group, rope_cols, dk, rope, norm_max=None):
    """``norm_max``: a zeroed fp32 [rope_cols / dk] buffer that receives, per rotated head, the
    largest row norm of the stored bf16 values (a by-product of the epilogue)."""
    return QKVRopeFn.apply(x, group, rope_cols, dk, rope, norm_max, *group.params)


# ============================================================================ polynomial attention
KIND_ID = {"signed_product": 0, "offset_square": 1, "lower_degree_mix": 2}


def attention_tables(doc_ids: torch.Tensor):
    """int32 position-in-document, document id and exclusive document end for every token."""
    from ..models.attention import doc_positions
    B, T = doc_ids.shape
    pos = doc_positions(doc_ids)
    t = torch.arange(T, device=doc_ids.device).expand(B, T)
    last = torch.ones_like(doc_ids, dtype=torch.bool)
    last[:, :-1] = doc_ids[:, 1:] != doc_ids[:, :-1]
    end_here = torch.where(last, t + 1, torch.full_like(t, T))
    doc_end = end_here.flip(-1).cummin(-1).values.flip(-1)
    return {"pos": pos, "pos32": pos.to(torch.int32).contiguous().view(-1),
            "doc32": doc_ids.to(torch.int32).contiguous().view(-1),
            "doc_end32": doc_end.to(torch.int32).contiguous().view(-1), "B": B, "T": T}


class PolyAttentionFn(torch.autograd.Function):
    """y [N, H*dv] = polynomial attention of the fused qkv buffer (see csrc/attn)."""

    @staticmethod
    def forward(ctx, qkv, kpar, kind, dk, dv, H, cols, tables, row_scale, rope=None):
        kid = KIND_ID[kind]
        par = torch.zeros(H, 4, device=qkv.device, dtype=torch.float32)
        if kind == "offset_square":
            par[:, 0] = kpar.detach().float()
        elif kind == "lower_degree_mix":
            par.copy_(kpar.detach().float())
        y = lib().poly_fwd(kid, dk, dv, qkv, list(cols), tables["pos32"], tables["doc32"], row_scale, par,
                           tables["B"], tables["T"], H)
        ctx.save_for_backward(qkv, par, row_scale)
        ctx.meta = (kind, kid, dk, dv, H, list(cols), tables, kpar is not None, rope)
        return y

    @staticmethod
    def backward(ctx, dy):
        qkv, par, row_scale = ctx.saved_tensors
        kind, kid, dk, dv, H, cols, tables, has_par, rope = ctx.meta
        dqkv, dpar = lib().poly_bwd(kid, dk, dv, qkv, cols, dy.contiguous(), tables["pos32"], tables["doc32"],
                                    tables["doc_end32"], row_scale, par, tables["B"], tables["T"], H,
                                    rope["cos"] if rope else None, rope["sin"] if rope else None)
        dqkv._ttb_unrotated = rope is not None
        dk_par = None
        if has_par:
            g = dpar.view(tables["B"], H, -1, 4).sum(dim=(0, 2))  # fixed-order reduction
            dk_par = g[:, 0].clone() if kind == "offset_square" else g
        return dqkv, dk_par, None, None, None, None, None, None, None, None


def poly_attention(qkv, kpar, kind, dk, dv, H, cols, tables, row_scale, rope=None):
    """``rope``: the rotary tables the projection used; the backward then returns gradients
    w.r.t. the pre-rotation projections (the inverse rotation runs in its epilogues)."""
    return PolyAttentionFn.apply(qkv, kpar, kind, dk, dv, H, cols, tables, row_scale, rope)


# ============================================================================ bilinear MLP
class BilinearMLPFn(torch.autograd.Function):
    """out = residual + alpha * D((x L^T + bl) * (x R^T + br)) + alpha*bd  (mode 0)
    or with silu on the left factor (mode 1, the SwiGLU control).  x: bf16 [N, d]."""

    @staticmethod
    def forward(ctx, x, residual, bl, br, bd, g_l, g_r, g_d, alpha, mode, *weights):
        (wl, sl), (wr, sr) = g_l.operand(), g_r.operand()
        N, F_ = x.shape[0], wl.shape[0]
        h = torch.empty(N, F_, device=x.device, dtype=torch.bfloat16)
        l = torch.empty_like(h)
        r = torch.empty_like(h)
        with _launching((g_l, sl), (g_r, sr)):
            if (sl is None) != (sr is None):  # one factor still resident: copy the other one alone
                lib().gather_rows(wl if sl is not None else wr, [sl if sl is not None else sr])
                sl = sr = None
            lib().bilinear(x, wl, wr, bl, br, int(mode), h, l, r, _gathers(sl, sr) if sl is not None else None)
        wd, sd = g_d.operand()
        with _launching((g_d, sd)):
            if residual is not None:
                out = torch.empty(N, wd.shape[0], device=x.device, dtype=torch.float32)
                _mm(h, wd.t(), out, c=residual, alpha=alpha, beta=1.0, bias=bd, gather=_gathers(sd))
            else:
                out = torch.empty(N, wd.shape[0], device=x.device, dtype=torch.bfloat16)
                _mm(h, wd.t(), out, alpha=alpha, bias=bd, gather=_gathers(sd))
        ctx.save_for_backward(x, h, l, r)
        ctx.groups = (g_l, g_r, g_d)
        ctx.alpha, ctx.mode, ctx.has_res = alpha, mode, residual is not None
        ctx.has_bias = bl is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        x, h, l, r = ctx.saved_tensors
        g_l, g_r, g_d = ctx.groups
        g = _take_bf16(dout, ctx.alpha)
        wd = g_d.bf16()
        # dl and dr side by side in one [N, 2F] buffer, so that dx = [dl | dr] @ [L; R] is one
        # GEMM over the concatenated contraction (F a multiple of the 64-wide k-block), written in
        # bf16 like the input
        F_ = l.shape[1]
        concat = F_ % 64 == 0
        if concat:
            dlr = torch.empty(l.shape[0], 2 * F_, device=l.device, dtype=l.dtype)
            dl, dr = dlr[:, :F_], dlr[:, F_:]
        else:
            dl, dr = torch.empty_like(l), torch.empty_like(r)
        lib().bilinear_grad(g, wd, l, r, dl, dr, int(ctx.mode))
        grads_d = g_d.sink_grad(lambda out, beta: _mm(g.t(), h, out, c=out, beta=beta))
        dx = torch.empty_like(x)
        if concat:
            _mm(dlr, g_l.bf16(), dx, b2=g_r.bf16())
        else:
            part = _mm(dl, g_l.bf16(), torch.empty(dx.shape, device=dx.device, dtype=torch.float32))
            _mm(dr, g_r.bf16(), dx, c=part, beta=1.0)
        grads_l = g_l.sink_grad(lambda out, beta: _mm(dl.t(), x, out, c=out, beta=beta))
        grads_r = g_r.sink_grad(lambda out, beta: _mm(dr.t(), x, out, c=out, beta=beta))
        dres = dout if ctx.has_res else None
        dbl = dbr = dbd = None
        if ctx.has_bias:
            dbl, dbr, dbd = dl.float().sum(0), dr.float().sum(0), g.float().sum(0)
        return (dx, dres, dbl, dbr, dbd, None, None, None, None, None, *grads_l, *grads_r, *grads_d)


def bilinear_mlp(x, g_l, g_r, g_d, residual=None, alpha=1.0, mode=0, bl=None, br=None, bd=None):
    return BilinearMLPFn.apply(x, residual, bl, br, bd, g_l, g_r, g_d, float(alpha), int(mode),
                               *g_l.params, *g_r.params, *g_d.params)


# ============================================================================ embedding
class EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, group, weight):
        ctx.save_for_backward(idx)
        ctx.group = group
        return lib().embed_fwd(idx.contiguous().view(-1), weight.detach().contiguous())

    @staticmethod
    def backward(ctx, dx):
        (idx,) = ctx.saved_tensors
        dx = dx.contiguous().float()

        def compute(out, beta):
            if beta == 0.0:
                out.zero_()
            lib().embed_bwd(idx.contiguous().view(-1), dx, out)

        (g,) = ctx.group.sink_grad(compute)
        return None, None, g


def embedding(idx, group):
    return EmbeddingFn.apply(idx, group, group.params[0])


# ============================================================================ fused linear + CE
class LinearCEFn(torch.autograd.Function):
    """Summed cross-entropy of (alpha * x W[:V]^T) against targets (-100 ignored), chunked over rows.

    Forward keeps the per-row log-sum-exp and, while they fit in ``KEEP_LOGITS_BYTES``, the fp32
    logits its GEMM epilogue already holds (written warp-coalesced beside the online LSE): the
    backward then forms bf16 dlogits in one elementwise pass instead of recomputing every chunk's
    logits with a second GEMM.  Otherwise the backward recomputes them in the GEMM.  Either way
    dx = dlogits W and dW += dlogits^T x follow."""

    KEEP_LOGITS_BYTES = 8 << 30

    @staticmethod
    def forward(ctx, x, targets, group, V, alpha, chunk, weight):
        w16 = group.bf16()
        N = x.shape[0]
        Vp = w16.shape[0]
        lse = torch.empty(N, device=x.device, dtype=torch.float32)
        total = torch.zeros((), device=x.device, dtype=torch.float32)
        keep = N * Vp * 4 <= LinearCEFn.KEEP_LOGITS_BYTES and Vp % 4 == 0 and any(ctx.needs_input_grad)
        z = torch.empty(N, Vp, device=x.device, dtype=torch.float32) if keep else None
        for s in range(0, N, chunk):
            e = min(N, s + chunk)
            loss_rows, l = lib().ce_fwd(x[s:e], w16, int(V), float(alpha), targets[s:e],
                                        z[s:e] if keep else None)
            lse[s:e] = l
            total += loss_rows.sum()
        ctx.save_for_backward(x, targets, lse)
        ctx.group, ctx.V, ctx.alpha, ctx.chunk, ctx.z = group, V, alpha, chunk, z
        return total

    @staticmethod
    def backward(ctx, g):
        x, targets, lse = ctx.saved_tensors
        group, V, alpha, chunk, z = ctx.group, ctx.V, ctx.alpha, ctx.chunk, ctx.z
        ctx.z = None
        w16 = group.bf16()
        Vp = w16.shape[0]
        g32 = g.detach().float().reshape(1).contiguous()
        N = x.shape[0]
        dx = torch.empty(N, x.shape[1], device=x.device, dtype=torch.float32)
        dlog = torch.empty(min(chunk, N), Vp, device=x.device, dtype=torch.bfloat16)

        def compute(out, beta):
            # one sink call per backward: the chunk loop runs inside it, the first chunk's dW GEMM
            # may overwrite the buffer (beta = 0) and later chunks accumulate
            for s in range(0, N, chunk):
                e = min(N, s + chunk)
                d = dlog[: e - s]
                if z is not None:
                    lib().ce_bwd_from_logits(z[s:e], float(alpha), targets[s:e], lse[s:e], g32, d)
                else:
                    lib().ce_bwd_logits(x[s:e], w16, int(V), float(alpha), targets[s:e], lse[s:e], g32, d)
                _mm(d, w16, dx[s:e])
                _mm(d.t(), x[s:e], out, c=out, beta=beta if s == 0 else 1.0)

        (gw,) = group.sink_grad(compute)
        return dx, None, None, None, None, None, gw


def linear_cross_entropy(x, targets, group, V, alpha=1.0, chunk=8192):
    return LinearCEFn.apply(x.contiguous(), targets.contiguous().view(-1), group, int(V), float(alpha), int(chunk),
                            group.params[0])
