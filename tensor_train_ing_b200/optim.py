"""Optimizers: AdamW reference grouping and Muon (hidden matrices) + AdamW (everything else).

Semantics follow the reference platform (tnlm/optim.py:16-99):
  * ``hidden_matrix``: 2-D ``blocks.*.weight`` parameters; L, R, D, Q1/K1/Q2/K2/V/O stay separate
    logical matrices for the optimizer even though the fused kernels concatenate them for compute;
  * AdamW groups: hidden matrices (decayed, width/depth LR scaling) vs everything else;
  * ``MuonAdamW``: Muon on hidden matrices, AdamW on vocabulary weights and small parameters, with
    a ``{"muon": ..., "adamw": ...}`` state dict and every group carrying ``base_lr``.

``Muon`` is this framework's implementation of the public Muon method with PyTorch's update rule
(torch.optim.Muon: momentum lerp, Nesterov lerp, 5 quintic Newton-Schulz steps in bf16 with the
published coefficients (3.4445, -4.7750, 2.0315), decoupled decay, shape-adjusted LR) and the
same state layout (``momentum_buffer``).  On CUDA each Newton-Schulz step is three tcgen05 GEMMs
whose epilogues fuse the affine combinations (``B = b A + c A A``, ``X = a X + B X``).
"""
from __future__ import annotations

import math

import torch

NS_COEFFICIENTS = (3.4445, -4.7750, 2.0315)
NS_STEPS = 5
NS_EPS = 1e-7
MUON_LR_RULES = ("original", "match_rms_adamw", "spectral_unclamped", "none")


def hidden_matrix(name: str, p: torch.Tensor) -> bool:
    """Linear-map weights inside blocks (head scalars such as ``coef`` are 2-D but not matrices)."""
    return p.ndim == 2 and name.startswith("blocks.") and name.endswith(".weight")


def param_split(model, only: set[int] | None = None):
    """(hidden matrices, vocabulary matrices, small params); ``only`` restricts to parameter ids
    (the parameters a rank owns under sharded data parallelism)."""
    vocab_ids = {id(model.embed.weight), id(model.unembed.weight)}
    hidden, vocab, small = [], [], []
    for name, p in model.named_parameters():
        if not p.requires_grad or (only is not None and id(p) not in only):
            continue
        if id(p) in vocab_ids:
            vocab.append(p)
        elif hidden_matrix(name, p):
            hidden.append(p)
        else:
            small.append(p)
    return hidden, vocab, small


def muon_lr_ratio(rule: str | None, shape) -> float:
    """LR multiplier for a matrix of shape (fan_out, fan_in)."""
    A, B = shape[0], shape[1]
    if rule is None or rule == "original":
        return math.sqrt(max(1.0, A / B))
    if rule == "match_rms_adamw":
        return 0.2 * math.sqrt(max(A, B))
    if rule == "spectral_unclamped":
        return math.sqrt(A / B)
    if rule == "none":
        return 1.0
    raise ValueError(f"unknown Muon LR rule {rule!r}; expected one of {MUON_LR_RULES}")


def newton_schulz(g: torch.Tensor, steps: int = NS_STEPS, coefficients=NS_COEFFICIENTS, eps: float = NS_EPS):
    """Approximate orthogonalisation U S' V^T of a 2-D matrix (bf16), as in the public Muon method."""
    a, b, c = coefficients
    x = g.to(torch.bfloat16)
    transposed = g.shape[0] > g.shape[1]
    if transposed:
        x = x.t()
    x = x / x.norm().clamp(min=eps)
    if x.is_cuda and _fused_ns_ok(x):
        x = _newton_schulz_fused(x.contiguous(), steps, a, b, c)
    else:
        for _ in range(steps):
            gram = x @ x.t()
            update = torch.addmm(gram, gram, gram, beta=b, alpha=c)
            x = torch.addmm(x, update, x, beta=a)
    return x.t() if transposed else x


def _fused_ns_ok(x):
    m, n = x.shape
    return m % 8 == 0 and n % 8 == 0


def _newton_schulz_fused(x, steps, a, b, c):
    from .ops._ext import lib
    C = lib()
    m, n = x.shape
    gram = torch.empty(m, m, device=x.device, dtype=torch.bfloat16)
    upd = torch.empty_like(gram)
    nxt = torch.empty_like(x)
    for _ in range(steps):
        C.mm(x, x.t(), gram)                                  # A = X X^T
        C.mm(gram, gram, upd, gram, float(c), float(b))       # B = c A A + b A
        C.mm(upd, x, nxt, x, 1.0, float(a))                   # X = B X + a X
        x, nxt = nxt, x
    return x


class Muon(torch.optim.Optimizer):
    """Muon for 2-D parameters (state: ``momentum_buffer``)."""

    def __init__(self, params, lr=1e-3, weight_decay=0.1, momentum=0.95, nesterov=True,
                 ns_coefficients=NS_COEFFICIENTS, eps=NS_EPS, ns_steps=NS_STEPS, adjust_lr_fn=None):
        if lr < 0 or momentum < 0 or weight_decay < 0:
            raise ValueError("lr, momentum and weight_decay must be non-negative")
        if adjust_lr_fn is not None and adjust_lr_fn not in MUON_LR_RULES:
            raise ValueError(f"Adjust learning rate function {adjust_lr_fn} is not supported")
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                        ns_coefficients=tuple(ns_coefficients), eps=eps, ns_steps=ns_steps,
                        adjust_lr_fn=adjust_lr_fn)
        super().__init__(params, defaults)
        for group in self.param_groups:
            for p in group["params"]:
                if p.ndim != 2:
                    raise ValueError("Muon only supports 2-D parameters")

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr, wd, mom = group["lr"], group["weight_decay"], group["momentum"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                state = self.state[p]
                if "momentum_buffer" not in state:
                    state["momentum_buffer"] = torch.zeros_like(p.grad)
                buf = state["momentum_buffer"]
                buf.lerp_(p.grad, 1 - mom)
                update = p.grad.lerp(buf, mom) if group["nesterov"] else buf
                update = newton_schulz(update, group["ns_steps"], group["ns_coefficients"], group["eps"])
                p.mul_(1 - lr * wd)
                p.add_(update, alpha=-lr * muon_lr_ratio(group["adjust_lr_fn"], p.shape))
        return loss


class MuonAdamW(torch.optim.Optimizer):
    """Muon on hidden matrices plus AdamW on the rest, presented as one optimizer."""

    # Identity written into checkpoints: the reference platform's class of the same optimizer (same
    # updates and state layout), whose loader requires that exact name, so either framework resumes
    # the other's Muon runs.  This framework's loader accepts both names.
    checkpoint_class = "tnlm.optim.MuonAdamW"

    def __init__(self, model, *, lr, aux_lr, weight_decay, betas, momentum=0.95, nesterov=True,
                 adjust_lr_fn="match_rms_adamw", vocab_weight_decay=0.0, only=None):
        hidden, vocab, small = param_split(model, only)
        self.muon = Muon([{"params": hidden, "base_lr": lr, "kind": "muon"}], lr=lr, weight_decay=weight_decay,
                         momentum=momentum, nesterov=nesterov, adjust_lr_fn=adjust_lr_fn)
        groups = [{"params": vocab, "weight_decay": vocab_weight_decay, "base_lr": aux_lr, "kind": "adamw_vocab"},
                  {"params": small, "weight_decay": 0.0, "base_lr": aux_lr, "kind": "adamw_small"}]
        fused = torch.cuda.is_available() and all(p.is_cuda for g in groups for p in g["params"])
        # serial: only non-empty groups (the reference layout); sharded: every group on every rank
        self.adamw = torch.optim.AdamW(groups if only is not None else [g for g in groups if g["params"]], lr=aux_lr,
                                       betas=betas, fused=fused or None)
        # not calling Optimizer.__init__: the children own groups and state
        self.defaults = {}
        self._optimizer_step_pre_hooks, self._optimizer_step_post_hooks = {}, {}

    @property
    def param_groups(self):
        return self.muon.param_groups + self.adamw.param_groups

    @property
    def state(self):
        return {**self.muon.state, **self.adamw.state}

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("MuonAdamW does not take a closure")
        self.muon.step()
        self.adamw.step()

    def zero_grad(self, set_to_none: bool = True):
        self.muon.zero_grad(set_to_none)
        self.adamw.zero_grad(set_to_none)

    def state_dict(self):
        return {"muon": self.muon.state_dict(), "adamw": self.adamw.state_dict()}

    def load_state_dict(self, sd):
        self.muon.load_state_dict(sd["muon"])
        self.adamw.load_state_dict(sd["adamw"])


def _scaling_multiplier(model) -> float:
    mcfg = getattr(model, "cfg", None)
    mult = 1.0
    if mcfg is not None and mcfg.width_scaling_base:
        mult *= (mcfg.width_scaling_base / mcfg.d_model) ** mcfg.width_lr_exponent
    if mcfg is not None and mcfg.depth_scaling_base:
        mult *= (mcfg.depth_scaling_base / mcfg.layers) ** mcfg.depth_lr_exponent
    return mult


def make_optimizer(model, cfg, only: set[int] | None = None):
    """cfg: TrainConfig.  'adamw' = the reference grouping; 'muon' = MuonAdamW.  ``only``: build it
    over these parameter ids (a rank's owned parameters); group hyper-parameters are unchanged."""
    betas = (cfg.beta1, cfg.beta2)
    mult = _scaling_multiplier(model)
    if cfg.optimizer == "adamw":
        hidden, vocab, small = param_split(model, only)
        groups = [{"params": hidden, "weight_decay": cfg.weight_decay_hidden / mult, "base_lr": cfg.lr * mult,
                   "lr": cfg.lr * mult},
                  {"params": vocab + small, "weight_decay": 0.0, "base_lr": cfg.lr}]
        fused = torch.cuda.is_available() and all(p.is_cuda for p in model.parameters())
        return torch.optim.AdamW(groups, lr=cfg.lr, betas=betas, fused=fused or None)
    if cfg.optimizer == "muon":
        if mult != 1.0:
            raise NotImplementedError("width/depth LR scaling is defined for AdamW only; Muon uses its own shape scaling")
        return MuonAdamW(model, lr=cfg.lr, aux_lr=cfg.aux_adamw_lr or cfg.lr, weight_decay=cfg.weight_decay_hidden,
                         betas=betas, momentum=cfg.muon_momentum, adjust_lr_fn=cfg.muon_adjust_lr, only=only)
    raise ValueError(f"unknown optimizer {cfg.optimizer!r}")
