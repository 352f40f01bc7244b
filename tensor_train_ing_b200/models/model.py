"""Tensor-network language model: bilinear MLP + polynomial (softmax-free) attention, and the
SwiGLU + softmax control.

Fixed by compatibility with the reference (tnlm/model.py:16-259), and tested bit for bit on CPU:
the module tree and state-dict names (``embed``, ``blocks.{i}.attn.{q1,k1,q2,k2,v,o}``,
``blocks.{i}.{attn_in,attn_out,mlp_in,mlp_out}``, ``blocks.{i}.mlp.{l,r,d}``, ``final_norm``,
``unembed``), the order in which modules are built and weights drawn (so a seed gives the same
weights), and the order of the forward's operations (so gradients sum in the same order).

Two execution paths share the parameters:
  * the module path (plain PyTorch math of ``models.attention``): the oracle and the CPU path;
  * the fused path (CUDA tensors, ``attention_backend`` auto/cuda/triton): every hot op runs on the
    sm_100a kernels of ``tensor_train_ing_b200.ops`` (``ops/block.py`` drives it).  The residual
    stream stays fp32 as under the reference's bf16 autocast with fp32 parameters.
"""
from __future__ import annotations

import warnings

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from .attention import (apply_rope, doc_positions, polynomial_attention, rope_tables, row_scale_mask,
                        softmax_attention, softmax_attention_flex, visible_mask)
from .normalization import SpectralLinear, make_norm

# normalization package -> (input norm kind, output norm kind, spectral linears)
PACKAGES = {
    "pre_rms": ("rms", None, False),
    "branch_rms": (None, "rms", False),
    "sandwich_rms": ("rms", "rms", False),
    "group_rms": ("group", None, False),
    "spectral_rms": ("rms", None, True),
    "lagged": ("lagged", None, False),
    "taper": ("taper", None, False),
}
# operator classes from least to most general: polynomial, normalised, general (softmax / SiLU)
CLASS_ORDER = {"P": 0, "N": 1, "G": 2}
ATTN_KIND_ID = {"signed_product": 0, "offset_square": 1, "lower_degree_mix": 2}
# attention kind -> number of (query, key) pairs: S = S1 (one pair) or a polynomial of S1 and S2
QK_PAIRS = {"softmax": 1, "offset_square": 1, "signed_product": 2, "lower_degree_mix": 2}


def _linear(d_in, d_out, spectral, bias=False):
    return SpectralLinear(d_in, d_out, bias) if spectral else nn.Linear(d_in, d_out, bias=bias)


def linear_weight(lin: nn.Module) -> torch.Tensor:
    """The matrix a linear layer applies (the effective weight for SpectralLinear)."""
    return lin.effective_weight() if isinstance(lin, SpectralLinear) else lin.weight


@torch.no_grad()
def score_bound(q: torch.Tensor, k: torch.Tensor, d_key: int) -> torch.Tensor:
    """Per head, max_i |q_i| * max_j |k_j| / sqrt(dk): by Cauchy-Schwarz never below the largest
    |S_ij| of the batch, whatever the mask (RoPE keeps norms).  q, k: (B, H, T, dk) -> (H,)."""
    top = lambda t: t.detach().float().norm(dim=-1).amax(dim=(0, 2))  # noqa: E731
    return top(q) * top(k) / d_key ** 0.5


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, spectral: bool):
        super().__init__()
        self.cfg, self.kind = cfg, cfg.attention
        self.record_score_bound, self.last_score_bound = False, None
        H, dk, dv, d = cfg.heads, cfg.d_key, cfg.d_value, cfg.d_model
        pairs = QK_PAIRS[self.kind]
        # built (and their spectral vectors drawn) in this order: q1, k1, [q2, k2], v, o
        for i in range(1, pairs + 1):
            setattr(self, f"q{i}", _linear(d, H * dk, spectral))
            setattr(self, f"k{i}", _linear(d, H * dk, spectral))
        self.v = _linear(d, H * dv, spectral)
        self.o = _linear(H * dv, d, spectral)
        if self.kind == "offset_square":
            self.b = nn.Parameter(torch.full((H,), cfg.offset_square_b))
        elif self.kind == "lower_degree_mix":  # (c0, c1, c2, c12): starts as the signed product S1 S2
            self.coef = nn.Parameter(torch.tensor([[0.0, 0.0, 0.0, 1.0]]).repeat(H, 1))
        default_power = 1.0 if self.kind == "offset_square" else 0.5
        self.row_power = default_power if cfg.attn_row_power is None else cfg.attn_row_power

    @property
    def op_class(self):
        return "G" if self.kind == "softmax" else "P"

    def qk_pairs(self) -> list[tuple[nn.Module, nn.Module]]:
        return [(getattr(self, f"q{i}"), getattr(self, f"k{i}")) for i in range(1, QK_PAIRS[self.kind] + 1)]

    def projections(self):
        """Linear layers whose outputs form the fused QKV buffer, in buffer order."""
        return [lin for pair in self.qk_pairs() for lin in pair] + [self.v]

    def _split_heads(self, x, lin, dh):
        B, T, _ = x.shape
        return lin(x).view(B, T, self.cfg.heads, dh).transpose(1, 2)

    def _mix_polynomial(self, x, ctx, q1, k1, q2, k2, v):
        cfg = self.cfg
        if self.record_score_bound:
            self.last_score_bound = {name: score_bound(q, k, cfg.d_key)
                                     for name, q, k in (("S1", q1, k1), ("S2", q2, k2)) if q is not None}
        if cfg.fp32_scores:  # at least fp32 (an fp64 oracle stays fp64)
            widen = lambda t: None if t is None else t.to(torch.promote_types(t.dtype, torch.float32))  # noqa: E731
            q1, k1, q2, k2, v = (widen(t) for t in (q1, k1, q2, k2, v))
        with torch.autocast(x.device.type, enabled=False):
            if ctx["backend"] == "recurrent":
                from .long_context import chunked_polynomial_attention
                y, _, _ = chunked_polynomial_attention(self.kind, q1, k1, q2, k2, v, ctx["doc_ids"],
                                                       ctx["row_scale"][self.row_power],
                                                       coef=getattr(self, "coef", None), b=getattr(self, "b", None))
            else:
                y = polynomial_attention(self.kind, q1, k1, q2, k2, v, ctx["C"][self.row_power],
                                         coef=getattr(self, "coef", None), b=getattr(self, "b", None))
        return y.to(x.dtype)

    def forward(self, x, ctx):
        """Module path: dense polynomial attention, or SDPA / FlexAttention for the softmax control."""
        cfg = self.cfg
        cos, sin = ctx["rope"]
        rotated = lambda lin: apply_rope(self._split_heads(x, lin, cfg.d_key), cos, sin)  # noqa: E731
        q1, k1 = rotated(self.q1), rotated(self.k1)
        v = self._split_heads(x, self.v, cfg.d_value)
        if self.kind == "softmax":
            y = (softmax_attention_flex(q1, k1, v, ctx["doc_ids"]) if ctx["backend"] == "flex"
                 else softmax_attention(q1, k1, v, ctx["visible"]))
        else:
            q2, k2 = (rotated(self.q2), rotated(self.k2)) if QK_PAIRS[self.kind] == 2 else (None, None)
            y = self._mix_polynomial(x, ctx, q1, k1, q2, k2, v)
        B, H, T, dv = y.shape
        return self.o(y.transpose(1, 2).reshape(B, T, H * dv))


class MLP(nn.Module):
    """``d(l(x) * r(x))``: bilinear (optionally with biases) or, for the control, SwiGLU."""

    def __init__(self, cfg: ModelConfig, spectral: bool):
        super().__init__()
        self.kind = cfg.mlp
        bias = self.kind == "affine_bilinear"
        self.l = _linear(cfg.d_model, cfg.d_mlp, spectral, bias)
        self.r = _linear(cfg.d_model, cfg.d_mlp, spectral, bias)
        self.d = _linear(cfg.d_mlp, cfg.d_model, spectral, bias)

    @property
    def op_class(self):
        return "G" if self.kind == "swiglu" else "P"

    def forward(self, x):
        gate = self.l(x)
        if self.kind == "swiglu":
            gate = F.silu(gate)
        return self.d(gate * self.r(x))


class Block(nn.Module):
    """Two residual branches, ``x + alpha * out_norm(branch(in_norm(x)))``, for attention then MLP;
    ``ablate`` (analysis only) removes whole branches."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        nin, nout, spectral = PACKAGES[cfg.normalization]
        self.alpha = cfg.residual_alpha
        if cfg.depth_residual_base:
            self.alpha *= (cfg.depth_residual_base / cfg.layers) ** cfg.depth_residual_exponent
        self.attn, self.mlp = Attention(cfg, spectral), MLP(cfg, spectral)
        norm = lambda kind: make_norm(kind, cfg.d_model, cfg) if kind else nn.Identity()  # noqa: E731
        self.attn_in, self.attn_out = norm(nin), norm(nout)
        self.mlp_in, self.mlp_out = norm(nin), norm(nout)
        self.ablate: frozenset = frozenset()

    def _residual(self, x, norm_in, branch, norm_out):
        return x + self.alpha * norm_out(branch(norm_in(x)))

    def forward(self, x, ctx):
        if self.ablate and self.training:
            raise RuntimeError("Block.ablate is analysis-only; reset it before training")
        if ctx.get("fused"):
            from ..ops.block import block_forward
            return block_forward(self, x, ctx)
        if "attn" not in self.ablate:
            x = self._residual(x, self.attn_in, lambda h: self.attn(h, ctx), self.attn_out)
        if "mlp" not in self.ablate:
            x = self._residual(x, self.mlp_in, self.mlp, self.mlp_out)
        return x


# Initialisation, one top-level component at a time in the draw order of the whole model (embedding,
# blocks in order, unembedding), so that a parameter-sharded model can stream the serial
# initialisation component by component (models/init_stream.py).
@torch.no_grad()
def init_embedding(embed: nn.Module):
    nn.init.normal_(embed.weight, std=1.0)


@torch.no_grad()
def init_block(blk: nn.Module, cfg: ModelConfig):
    """Inputs maps (Q, K, V, L, R): std fan_in^-1/2, queries and keys then times ``qk_init_scale``;
    output maps (O, D): std (2 depth fan_in)^-1/2; biases 0; spectral gains = sigma(W)."""
    a, m = blk.attn, blk.mlp
    extra_qk = [a.q2, a.k2] if QK_PAIRS[a.kind] == 2 else []
    for lin in [a.q1, a.k1, a.v, m.l, m.r] + extra_qk:  # the draw order
        nn.init.normal_(lin.weight, std=lin.weight.shape[1] ** -0.5)
    if cfg.qk_init_scale != 1.0:  # scores scale by s^2 per factor
        for lin in [a.q1, a.k1] + extra_qk:
            lin.weight.mul_(cfg.qk_init_scale)
    depth = cfg.depth_residual_base or cfg.layers
    for lin in (a.o, m.d):
        nn.init.normal_(lin.weight, std=(2 * depth * lin.weight.shape[1]) ** -0.5)
    for mod in blk.modules():
        if isinstance(mod, (nn.Linear, SpectralLinear)) and mod.bias is not None:
            mod.bias.zero_()
        if isinstance(mod, SpectralLinear):
            mod.reset_gamma()


@torch.no_grad()
def init_unembedding(unembed: nn.Module):
    nn.init.normal_(unembed.weight, std=0.02)


def operator_classes(model: nn.Module) -> dict:
    """Every module that declares an operator class, by name (the root is "<root>")."""
    out = {}
    for name, mod in model.named_modules():
        cls = getattr(mod, "op_class", None)
        if isinstance(cls, str):
            out[name or "<root>"] = cls
    return out


class TensorLM(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.padded_vocab, cfg.d_model)
        self.blocks = nn.ModuleList(Block(cfg) for _ in range(cfg.layers))
        self.final_norm = make_norm(cfg.final_normalization, cfg.d_model, cfg)
        self.unembed = nn.Linear(cfg.d_model, cfg.padded_vocab, bias=False)
        if cfg.tie_embeddings:
            self.unembed.weight = self.embed.weight
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        init_embedding(self.embed)
        for blk in self.blocks:
            init_block(blk, self.cfg)
        if not self.cfg.tie_embeddings:
            init_unembedding(self.unembed)

    @property
    def logit_multiplier(self) -> float:
        c = self.cfg
        return (c.width_scaling_base / c.d_model) ** c.width_logit_exponent if c.width_scaling_base else 1.0

    # ---------------------------------------------------------------- structure reports
    def operator_audit(self) -> dict:
        """The model's operator class is its most general node's ("P" < "N" < "G")."""
        nodes = operator_classes(self)
        worst = max(nodes.values(), key=lambda c: CLASS_ORDER[c], default="P")
        return {"class": worst, "nodes": nodes}

    def param_counts(self) -> dict:
        sizes = {"total": 0, "matrices": 0}
        for p in self.parameters():  # tied weights once
            sizes["total"] += p.numel()
        for _, p in self.named_parameters():
            if p.dim() >= 2:
                sizes["matrices"] += p.numel()
        vocab = self.embed.weight.numel() + (0 if self.cfg.tie_embeddings else self.unembed.weight.numel())
        return {**sizes, "non_embedding_matrices": sizes["matrices"] - vocab,
                "small": sizes["total"] - sizes["matrices"]}

    # ---------------------------------------------------------------- execution path
    def _row_powers(self) -> tuple:
        powers = {0.5, 1.0}
        if self.cfg.attn_row_power is not None:
            powers.add(self.cfg.attn_row_power)
        return tuple(sorted(powers))

    def fused_path_supported(self) -> tuple[bool, str]:
        """Shapes the sm_100a kernels cover: head dims 64/128, TMA-aligned widths, d_model <= 8192."""
        c = self.cfg
        if c.attention == "softmax":
            return False, "softmax control runs on PyTorch attention"
        if c.d_key not in (64, 128) or c.d_value not in (64, 128):
            return False, f"head dims {c.d_key}/{c.d_value} (kernels cover 64 and 128)"
        if c.d_model % 64 or c.d_mlp % 8 or c.padded_vocab % 8 or c.d_model > 8192:
            return False, "d_model must be a multiple of 64 (<= 8192); d_mlp and padded_vocab multiples of 8"
        return True, ""

    def uses_fused_path(self, idx: torch.Tensor) -> bool:
        backend = self.cfg.attention_backend
        if getattr(self, "_force_reference", False):  # module hooks (analysis, calibration) need the module path
            return False
        if not (idx.is_cuda and backend in ("auto", "cuda", "triton")):
            return False
        ok, why = self.fused_path_supported()
        if ok:
            return True
        if backend != "auto":
            raise ValueError(f"attention_backend={backend!r} needs the fused kernels, which do not cover: {why}")
        if not getattr(self, "_warned_fused", False):
            warnings.warn(f"TensorLM: using the PyTorch module path ({why})")
            self._warned_fused = True
        return False

    def make_ctx(self, idx, doc_ids):
        """Per-batch tables: document positions, RoPE, and the backend's masks or row scales."""
        if doc_ids is None:
            doc_ids = torch.zeros(idx.shape, dtype=torch.long, device=idx.device)
        pos = doc_positions(doc_ids)
        ctx = {"doc_ids": doc_ids}
        if self.uses_fused_path(idx):
            from ..ops.block import fused_context
            ctx.update(fused_context(self, doc_ids, pos))
            return ctx
        ctx["rope"] = rope_tables(pos, self.cfg.d_key, self.cfg.rope_base)
        backend = self.cfg.attention_backend
        if backend == "auto":
            backend = "triton" if idx.is_cuda else "reference"
        if self.cfg.attention == "softmax":
            backend = "flex" if backend in ("triton", "cuda") else "softmax"
        ctx["backend"] = backend
        if backend == "recurrent":  # the linear-state form needs row scales, never a T x T mask
            if self.cfg.attention == "softmax":
                raise ValueError("the recurrent attention backend has no softmax form")
            scale = lambda p: torch.where(doc_ids >= 0, (pos + 1).to(torch.float64).pow(-p), 0.0)  # noqa: E731
            ctx["row_scale"] = {p: scale(p) for p in self._row_powers()}
            return ctx
        if backend != "flex":  # the dense paths; FlexAttention builds its own block mask
            ctx["visible"] = visible_mask(doc_ids)
            if self.cfg.attention != "softmax":
                ctx["C"] = {p: row_scale_mask(ctx["visible"], p) for p in self._row_powers()}
        return ctx

    # ---------------------------------------------------------------- forward (module path)
    def recomputed_blocks(self) -> int:
        """How many blocks (the first ones) a training forward recomputes in backward under
        activation checkpointing: all of them, unless ``recompute_blocks`` (set by the training engine
        when the device has room to keep some blocks' activations) says fewer.  Keeping the last
        blocks' activations changes no value, only memory and time."""
        if not (self.cfg.activation_checkpointing and self.training and torch.is_grad_enabled()):
            return 0
        limit = getattr(self, "recompute_blocks", None)
        n = len(self.blocks)
        return n if limit is None else max(0, min(n, int(limit)))

    def _trunk(self, idx, ctx):
        x = self.embed(idx)
        recompute = self.recomputed_blocks()
        for i, blk in enumerate(self.blocks):
            x = torch.utils.checkpoint.checkpoint(blk, x, ctx, use_reentrant=False) if i < recompute else blk(x, ctx)
        return self.final_norm(x)

    def _loss(self, x, targets):
        """(logits or None, summed cross-entropy) over the real vocabulary (padded rows never score)."""
        V = self.cfg.vocab_size
        scaled = self.cfg.width_scaling_base
        if self.cfg.loss_chunk_tokens > 0:
            from ..ops.linear_ce import chunked_linear_cross_entropy_reference
            w = self.unembed.weight[:V]
            if scaled:
                w = w * self.logit_multiplier
            return None, chunked_linear_cross_entropy_reference(x.flatten(0, 1), w, targets.flatten(),
                                                                self.cfg.loss_chunk_tokens)
        logits = self.unembed(x)[..., :V]
        if scaled:
            logits = logits * self.logit_multiplier
        wide = logits.to(torch.promote_types(logits.dtype, torch.float32))
        return logits, F.cross_entropy(wide.flatten(0, 1), targets.flatten(), ignore_index=-100, reduction="sum")

    def forward(self, idx, doc_ids=None, targets=None, reduction="mean"):
        """Logits (no targets), else (logits or None, loss sum, valid targets) for ``reduction="sum"``
        or (logits or None, mean loss)."""
        ctx = self.make_ctx(idx, doc_ids)
        if ctx.get("fused"):
            from ..ops.block import model_forward
            return model_forward(self, idx, ctx, targets, reduction)
        if getattr(self, "_ttb_weights_remote", False):
            raise RuntimeError("this parameter-sharded model holds non-owned weights only as the fused path's bf16 "
                               "caches; the module path cannot run it")
        x = self._trunk(idx, ctx)
        if targets is None:
            logits = self.unembed(x)[..., :self.cfg.vocab_size]
            return logits * self.logit_multiplier if self.cfg.width_scaling_base else logits
        logits, loss = self._loss(x, targets)
        n = (targets != -100).sum()
        return (logits, loss, n) if reduction == "sum" else (logits, loss / n.clamp_min(1))
