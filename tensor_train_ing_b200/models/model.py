"""Tensor-network language model: bilinear MLP + polynomial (softmax-free) attention, and the
SwiGLU + softmax control.

The module tree and state-dict names are the reference's (tnlm/model.py:16-259):
``embed``, ``blocks.{i}.attn.{q1,k1,q2,k2,v,o}``, ``blocks.{i}.{attn_in,attn_out,mlp_in,mlp_out}``,
``blocks.{i}.mlp.{l,r,d}``, ``final_norm``, ``unembed`` -- so reference checkpoints load as is.

Two execution paths share the parameters:
  * the *reference* path: plain PyTorch math (``models.attention``) -- the oracle, and the CPU path;
  * the *fused* path (CUDA tensors, ``attention_backend`` in auto/cuda/triton): every hot op runs on
    the hand-written sm_100a kernels of ``tensor_train_ing_b200.ops`` -- RMSNorm producing bf16,
    one QKV GEMM with a RoPE epilogue, tcgen05 polynomial attention, output GEMM with a fused
    residual add, dual-B bilinear GEMM, down GEMM with fused residual, fused chunked linear-CE.
    The residual stream stays fp32 as under the reference's bf16 autocast with fp32 parameters.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig
from .attention import (apply_rope, doc_positions, polynomial_attention, rope_tables, row_scale_mask,
                        row_scale_vector, softmax_attention, softmax_attention_flex, visible_mask)
from .normalization import GroupRMSNorm, LaggedRMS, RMSNorm, SpectralLinear, TaperRMS, make_norm

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
CLASS_ORDER = {"P": 0, "N": 1, "G": 2}
ATTN_KIND_ID = {"signed_product": 0, "offset_square": 1, "lower_degree_mix": 2}


def _linear(d_in, d_out, spectral, bias=False):
    return SpectralLinear(d_in, d_out, bias) if spectral else nn.Linear(d_in, d_out, bias=bias)


def linear_weight(lin: nn.Module) -> torch.Tensor:
    """The matrix a linear layer applies (the effective weight for SpectralLinear)."""
    return lin.effective_weight() if isinstance(lin, SpectralLinear) else lin.weight


@torch.no_grad()
def score_bound(q: torch.Tensor, k: torch.Tensor, d_key: int) -> torch.Tensor:
    """Per-head Cauchy-Schwarz bound max|q| * max|k| / sqrt(dk) on |S| over a batch (never below
    the true masked maximum; RoPE preserves norms).  q, k: (B, H, T, dk)."""
    qn = q.detach().float().norm(dim=-1).amax(dim=(0, 2))
    kn = k.detach().float().norm(dim=-1).amax(dim=(0, 2))
    return qn * kn / d_key ** 0.5


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, spectral: bool):
        super().__init__()
        self.cfg, self.kind = cfg, cfg.attention
        self.record_score_bound, self.last_score_bound = False, None
        H, dk, dv, d = cfg.heads, cfg.d_key, cfg.d_value, cfg.d_model
        self.q1 = _linear(d, H * dk, spectral)
        self.k1 = _linear(d, H * dk, spectral)
        if self.kind in ("signed_product", "lower_degree_mix"):
            self.q2 = _linear(d, H * dk, spectral)
            self.k2 = _linear(d, H * dk, spectral)
        self.v = _linear(d, H * dv, spectral)
        self.o = _linear(H * dv, d, spectral)
        if self.kind == "offset_square":
            self.b = nn.Parameter(torch.full((H,), cfg.offset_square_b))
        if self.kind == "lower_degree_mix":
            self.coef = nn.Parameter(torch.tensor([[0.0, 0.0, 0.0, 1.0]]).repeat(H, 1))
        default_power = 1.0 if self.kind == "offset_square" else 0.5
        self.row_power = default_power if cfg.attn_row_power is None else cfg.attn_row_power

    @property
    def op_class(self):
        return "G" if self.kind == "softmax" else "P"

    def projections(self):
        """Linear layers whose outputs form the fused QKV buffer, in buffer order."""
        names = ["q1", "k1"] + (["q2", "k2"] if hasattr(self, "q2") else []) + ["v"]
        return [getattr(self, n) for n in names]

    def _heads(self, x, lin, dh):
        B, T, _ = x.shape
        return lin(x).view(B, T, self.cfg.heads, dh).transpose(1, 2)

    def forward(self, x, ctx):
        """Reference path (dense oracle math, or FlexAttention for the softmax control)."""
        cfg = self.cfg
        cos, sin = ctx["rope"]
        q1 = apply_rope(self._heads(x, self.q1, cfg.d_key), cos, sin)
        k1 = apply_rope(self._heads(x, self.k1, cfg.d_key), cos, sin)
        v = self._heads(x, self.v, cfg.d_value)
        if self.kind == "softmax":
            if ctx["backend"] == "flex":
                y = softmax_attention_flex(q1, k1, v, ctx["doc_ids"])
            else:
                y = softmax_attention(q1, k1, v, ctx["visible"])
        else:
            q2 = k2 = None
            if hasattr(self, "q2"):
                q2 = apply_rope(self._heads(x, self.q2, cfg.d_key), cos, sin)
                k2 = apply_rope(self._heads(x, self.k2, cfg.d_key), cos, sin)
            if self.record_score_bound:
                self.last_score_bound = {name: score_bound(q, k, cfg.d_key)
                                         for name, q, k in (("S1", q1, k1), ("S2", q2, k2)) if q is not None}
            if cfg.fp32_scores:
                up = lambda t: None if t is None else t.to(torch.promote_types(t.dtype, torch.float32))
                q1, k1, q2, k2, v = map(up, (q1, k1, q2, k2, v))
            C = ctx["C"][self.row_power]
            with torch.autocast(x.device.type, enabled=False):
                y = polynomial_attention(self.kind, q1, k1, q2, k2, v, C,
                                         coef=getattr(self, "coef", None), b=getattr(self, "b", None))
            y = y.to(x.dtype)
        B, H, T, dv = y.shape
        return self.o(y.transpose(1, 2).reshape(B, T, H * dv))


class MLP(nn.Module):
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
        if self.kind == "swiglu":
            return self.d(F.silu(self.l(x)) * self.r(x))
        return self.d(self.l(x) * self.r(x))


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        nin, nout, spectral = PACKAGES[cfg.normalization]
        self.alpha = cfg.residual_alpha
        if cfg.depth_residual_base:
            self.alpha *= (cfg.depth_residual_base / cfg.layers) ** cfg.depth_residual_exponent
        self.attn, self.mlp = Attention(cfg, spectral), MLP(cfg, spectral)
        mk = lambda kind: make_norm(kind, cfg.d_model, cfg) if kind else nn.Identity()
        self.attn_in, self.attn_out = mk(nin), mk(nout)
        self.mlp_in, self.mlp_out = mk(nin), mk(nout)
        self.ablate: frozenset = frozenset()

    def forward(self, x, ctx):
        if self.ablate and self.training:
            raise RuntimeError("Block.ablate is analysis-only; reset it before training")
        if ctx.get("fused"):
            from ..ops.block import block_forward
            return block_forward(self, x, ctx)
        if "attn" not in self.ablate:
            x = x + self.alpha * self.attn_out(self.attn(self.attn_in(x), ctx))
        if "mlp" not in self.ablate:
            x = x + self.alpha * self.mlp_out(self.mlp(self.mlp_in(x)))
        return x


# Initialisation of each top-level component, in the order TensorLM.reset_parameters draws them
# (reference tnlm/model.py reset_parameters).  Kept per component so that a sharded model can stream
# the serial initialisation one component at a time (models/init_stream.py).
@torch.no_grad()
def init_embedding(embed: nn.Module):
    nn.init.normal_(embed.weight, std=1.0)


@torch.no_grad()
def init_block(blk: nn.Module, cfg: ModelConfig):
    a, m = blk.attn, blk.mlp
    for lin in [a.q1, a.k1, a.v, m.l, m.r] + ([a.q2, a.k2] if hasattr(a, "q2") else []):
        nn.init.normal_(lin.weight, std=lin.weight.shape[1] ** -0.5)
    if cfg.qk_init_scale != 1.0:
        for lin in [a.q1, a.k1] + ([a.q2, a.k2] if hasattr(a, "q2") else []):
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
        """Fan-in init: embed N(0,1); Q/K/V/L/R std fan_in^-1/2 (Q/K times qk_init_scale);
        O/D std (2*depth*fan_in)^-1/2; unembed 0.02; biases 0; spectral gamma = sigma(W).
        The draw order matches the reference so a seed gives identical weights."""
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
        classes = {}
        for name, mod in self.named_modules():
            c = getattr(mod, "op_class", None)
            if isinstance(c, str):
                classes[name or "<root>"] = c
        overall = max(classes.values(), key=CLASS_ORDER.get) if classes else "P"
        return {"class": overall, "nodes": classes}

    def param_counts(self) -> dict:
        matrices = sum(p.numel() for _, p in self.named_parameters() if p.dim() >= 2)
        total = sum(p.numel() for p in self.parameters())
        emb = self.embed.weight.numel() + (0 if self.cfg.tie_embeddings else self.unembed.weight.numel())
        return {"total": total, "matrices": matrices, "non_embedding_matrices": matrices - emb,
                "small": total - matrices}

    # ---------------------------------------------------------------- forward
    def _row_powers(self) -> tuple:
        extra = {self.cfg.attn_row_power} if self.cfg.attn_row_power is not None else set()
        return tuple(sorted({0.5, 1.0} | extra))

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
        if getattr(self, "_force_reference", False):  # analysis hooks need the module-level path
            return False
        if not (idx.is_cuda and backend in ("auto", "cuda", "triton")):
            return False
        ok, why = self.fused_path_supported()
        if not ok:
            if backend != "auto":
                raise ValueError(f"attention_backend={backend!r} needs the fused kernels, which do not cover: {why}")
            if not getattr(self, "_warned_fused", False):
                import warnings
                warnings.warn(f"TensorLM: using the PyTorch reference path ({why})")
                self._warned_fused = True
            return False
        return True

    def make_ctx(self, idx, doc_ids):
        B, T = idx.shape
        if doc_ids is None:
            doc_ids = torch.zeros(B, T, dtype=torch.long, device=idx.device)
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
        if backend != "flex":
            vis = visible_mask(doc_ids)
            ctx["visible"] = vis
            if self.cfg.attention != "softmax":
                ctx["C"] = {p: row_scale_mask(vis, p) for p in self._row_powers()}
        return ctx

    def forward(self, idx, doc_ids=None, targets=None, reduction="mean"):
        ctx = self.make_ctx(idx, doc_ids)
        if ctx.get("fused"):
            from ..ops.block import model_forward
            return model_forward(self, idx, ctx, targets, reduction)
        if getattr(self, "_ttb_weights_remote", False):
            raise RuntimeError("this parameter-sharded model holds non-owned weights only as the fused path's bf16 "
                               "caches; the PyTorch reference path cannot run it")
        x = self.embed(idx)
        ckpt = self.cfg.activation_checkpointing and self.training and torch.is_grad_enabled()
        for blk in self.blocks:
            x = torch.utils.checkpoint.checkpoint(blk, x, ctx, use_reentrant=False) if ckpt else blk(x, ctx)
        x = self.final_norm(x)
        V = self.cfg.vocab_size
        if targets is not None and self.cfg.loss_chunk_tokens > 0:
            from ..ops.linear_ce import chunked_linear_cross_entropy_reference
            w = self.unembed.weight[:V]
            if self.cfg.width_scaling_base:
                w = w * self.logit_multiplier
            loss = chunked_linear_cross_entropy_reference(x.flatten(0, 1), w, targets.flatten(),
                                                          self.cfg.loss_chunk_tokens)
            logits = None
        else:
            logits = self.unembed(x)[..., :V]
            if self.cfg.width_scaling_base:
                logits = logits * self.logit_multiplier
            if targets is None:
                return logits
            loss = F.cross_entropy(logits.to(torch.promote_types(logits.dtype, torch.float32)).flatten(0, 1),
                                   targets.flatten(), ignore_index=-100, reduction="sum")
        n = (targets != -100).sum()
        if reduction == "sum":
            return logits, loss, n
        return logits, loss / n.clamp_min(1)
