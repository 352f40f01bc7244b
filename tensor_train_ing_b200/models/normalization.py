"""Normalisation modules and the spectral (sigma-reparameterised) linear map.

Module, parameter and buffer names are those of the reference (tnlm/normalization.py:15-381), so its
checkpoints load here, and the arithmetic is written with the same operations in the same order,
so CPU trajectories agree bit for bit:

  RMSNorm / GroupRMSNorm   weight                                         class "N"
  LaggedRMS                weight, mean_sq, calibrated                    class "P"
  TaperRMS                 weight, weight_tilde, gate, c, s_tgt,          "N" until frozen at gate 0
                           ema_num, ema_den, ema_r, ema_steps, frozen
  SpectralLinear           weight, [bias], gamma, u, v

Structure: ``DynamicNorm`` is an input-dependent divisor with analysis hooks (record / clamp / const);
``_StatNorm`` is the base of the two norms that learn statistics while training (a valid-token mask,
count-weighted accumulators summed across data-parallel ranks at commit); ``SpectralLinear`` keeps
its power-iteration vectors as buffers that only ``spectral_step`` advances.  On CUDA the fused
model path runs these norms on the kernels of ops/norms.py and the spectral weights on
csrc/misc/spectral.cu; the forwards here are the definition those are tested against.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

SIGMA_FLOOR = 1e-12
ANALYSIS_MODES = (None, "record", "clamp", "const")


def upcast(x: torch.Tensor) -> torch.Tensor:
    """Reduction dtype: fp32, or fp64 when the input already is fp64 (oracle tests)."""
    return x.to(torch.promote_types(x.dtype, torch.float32))


def _rms(xf: torch.Tensor, eps: float) -> torch.Tensor:
    return torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps)


def _scale_by(x, divisor, weight):
    return (upcast(x) / divisor * upcast(weight)).to(x.dtype)


# ------------------------------------------------------------------------------------ dynamic norms
class DynamicNorm(nn.Module):
    """``x / r(x) * weight`` with an input-dependent divisor r.  ``denom_mode`` (analysis only):
    "record" stores r, "clamp" reuses the stored r (finite-ablation decomposition), "const" uses
    ``denom_const`` (a fixed-denominator approximation); training always uses the live r."""

    op_class = "N"

    def __init__(self, d: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))
        self.denom_mode: str | None = None
        self.denom_saved: torch.Tensor | None = None
        self.denom_const: torch.Tensor | None = None

    def denom(self, x: torch.Tensor) -> torch.Tensor:  # pragma: no cover - abstract
        raise NotImplementedError

    def _divisor(self, x):
        mode = self.denom_mode
        if mode is not None and self.training:
            raise RuntimeError("denom_mode is analysis-only; reset it before training")
        r = self.denom(x)
        if mode == "record":
            self.denom_saved = r.detach()
        elif mode == "clamp":
            r = self.denom_saved.to(r.dtype)
        elif mode == "const":
            r = self.denom_const.to(device=r.device, dtype=r.dtype).expand_as(r)
        elif mode not in ANALYSIS_MODES:
            raise ValueError(f"unknown denom_mode {mode!r}")
        return r

    def forward(self, x):
        return _scale_by(x, self._divisor(x), self.weight)


class RMSNorm(DynamicNorm):
    def denom(self, x):
        return _rms(upcast(x), self.eps)


class GroupRMSNorm(DynamicNorm):
    """RMS over ``groups`` contiguous feature groups (one divisor per token and group)."""

    def __init__(self, d: int, groups: int = 4, eps: float = 1e-6):
        super().__init__(d, eps)
        if d % groups:
            raise ValueError(f"d_model {d} is not divisible into {groups} groups")
        self.groups = groups

    def denom(self, x):
        xg = upcast(x).unflatten(-1, (self.groups, -1))
        return _rms(xg, self.eps).expand_as(xg).flatten(-2)


# ------------------------------------------------------------------------------------ learned statistics
class _StatNorm(nn.Module):
    """A norm that accumulates statistics while ``collecting`` (padding excluded through the valid
    mask), folds them in once per optimizer step with ``commit`` (summed across data-parallel ranks
    first, so the buffers stay replicated) and must not run under activation recomputation while
    collecting (the recomputed forward would count twice)."""

    def __init__(self):
        super().__init__()
        self.collecting = False
        self._valid: torch.Tensor | None = None

    def set_valid_mask(self, valid: torch.Tensor | None):
        self._valid = valid

    def _accumulators(self) -> list[torch.Tensor]:  # pragma: no cover - abstract
        raise NotImplementedError

    def _sum_across_ranks(self, distributed: bool) -> torch.Tensor:
        stats = torch.stack(self._accumulators())
        if distributed and torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.all_reduce(stats)
        return stats

    def _clear(self):
        for acc in self._accumulators():
            acc.zero_()


class LaggedRMS(_StatNorm):
    """Divides by a detached scalar: ``x / sqrt(mean_sq + eps) * weight``, so a batch never affects its
    own output.  ``mean_sq`` is an EMA of the per-token mean square with a half-life in tokens; the
    first commit after calibration starts replaces it outright."""

    op_class = "P"

    def __init__(self, d: int, eps: float = 1e-6, half_life_tokens: float = 1e6):
        super().__init__()
        self.eps, self.half_life_tokens = eps, half_life_tokens
        self.weight = nn.Parameter(torch.ones(d))
        self.register_buffer("mean_sq", torch.ones((), dtype=torch.float64))
        self.register_buffer("calibrated", torch.zeros((), dtype=torch.bool))
        self.register_buffer("acc_sum", torch.zeros((), dtype=torch.float64), persistent=False)
        self.register_buffer("acc_count", torch.zeros((), dtype=torch.float64), persistent=False)

    def _accumulators(self):
        return [self.acc_sum, self.acc_count]

    def denom(self, x):
        # the square root in the fp64 statistic first: mean_sq = 1e60 still gives an fp32 divisor
        return torch.sqrt(self.mean_sq + self.eps).to(torch.promote_types(x.dtype, torch.float32))

    @torch.no_grad()
    def _observe(self, x):
        per_token = x.detach().double().pow(2).mean(-1)
        if self._valid is not None:
            per_token = per_token * self._valid
            tokens = self._valid.sum()
        else:
            tokens = torch.tensor(float(per_token.numel()), device=per_token.device, dtype=per_token.dtype)
        self.acc_sum += per_token.sum()
        self.acc_count += tokens

    def forward(self, x):
        if self.collecting:
            self._observe(x)
        return _scale_by(x, self.denom(x), self.weight)

    @torch.no_grad()
    def commit(self, distributed: bool = True) -> float:
        stats = self._sum_across_ranks(distributed)
        self.acc_sum.copy_(stats[0])
        self.acc_count.copy_(stats[1])
        tokens = float(self.acc_count)
        if tokens == 0:
            return float(self.mean_sq)
        batch_ms = self.acc_sum / self.acc_count
        if bool(self.calibrated):
            keep = 0.5 ** (tokens / self.half_life_tokens)
            self.mean_sq.mul_(keep).add_((1 - keep) * batch_ms)
        else:
            self.mean_sq.copy_(batch_ms)
            self.calibrated.fill_(True)
        self._clear()
        if not torch.isfinite(self.mean_sq):
            raise FloatingPointError("the lagged RMS statistic became non-finite")
        return float(self.mean_sq)


class TaperRMS(_StatNorm):
    """TaperNorm, RMS form: ``g * x/r(x) * weight + (1 - g) * c * x * weight_tilde``.

    g = 1 is RMSNorm; g = 0 is the fixed diagonal map ``c * weight_tilde`` (class "P"), which folds
    into the next linear map.  Lifecycle (driven by training_taper.TaperLifecycle): warm-up
    statistics at g = 1; ``freeze`` sets c = E[|x w|^2 / r] / E[|x w|^2] (the least-squares match of
    the linear branch to the normalised one), s_tgt = E[r] and weight_tilde = weight from the
    bias-corrected EMAs; then a shared gate decays 1 -> 0 while training accumulates the
    differentiable anchor (r - s_tgt)^2 that ``taper_anchor_loss`` reads."""

    _BUFFERS = (("gate", 1.0), ("c", 1.0), ("s_tgt", 1.0), ("ema_num", 0.0), ("ema_den", 0.0), ("ema_r", 0.0),
                ("ema_steps", 0.0))

    def __init__(self, d: int, eps: float = 1e-6, ema_rate: float = 0.01):
        super().__init__()
        self.eps, self.ema_rate = eps, ema_rate
        self.weight = nn.Parameter(torch.ones(d))
        self.weight_tilde = nn.Parameter(torch.ones(d))
        for name, init in self._BUFFERS:
            self.register_buffer(name, torch.tensor(init, dtype=torch.float64))
        self.register_buffer("frozen", torch.zeros((), dtype=torch.bool))
        for name in ("acc_num", "acc_den", "acc_r", "acc_count"):
            self.register_buffer(name, torch.zeros((), dtype=torch.float64), persistent=False)
        self._anchor_sum: torch.Tensor | None = None
        self._anchor_count = 0.0

    @property
    def op_class(self):
        return "P" if bool(self.frozen) and float(self.gate) == 0.0 else "N"

    def _accumulators(self):
        return [self.acc_num, self.acc_den, self.acc_r, self.acc_count]

    @torch.no_grad()
    def _observe(self, xf, r):
        sq = (xf.detach() * upcast(self.weight.detach())).double().pow(2).sum(-1)
        rr = r.detach().double().squeeze(-1)
        w = self._valid.double() if self._valid is not None else torch.ones_like(rr)
        self.acc_num += (sq / rr * w).sum()
        self.acc_den += (sq * w).sum()
        self.acc_r += (rr * w).sum()
        self.acc_count += w.sum()

    def _anchor(self, r):
        dev = (r.squeeze(-1) - self.s_tgt.to(r.dtype)).pow(2)
        if self._valid is not None:
            dev, tokens = dev * self._valid, float(self._valid.sum())
        else:
            tokens = float(dev.numel())
        total = dev.sum()
        self._anchor_sum = total if self._anchor_sum is None else self._anchor_sum + total
        self._anchor_count += tokens

    def forward(self, x):
        xf = upcast(x)
        g = float(self.gate)
        frozen = bool(self.frozen)
        anchored = self.training and frozen
        r = _rms(xf, self.eps) if (g > 0 or self.collecting or anchored) else None
        if self.collecting and not frozen:
            self._observe(xf, r)
        if anchored:
            self._anchor(r)
        linear = float(self.c) * xf * upcast(self.weight_tilde)
        if g == 0.0:
            return linear.to(x.dtype)
        normed = xf / r * upcast(self.weight)
        return (normed if g == 1.0 else g * normed + (1 - g) * linear).to(x.dtype)

    @torch.no_grad()
    def commit(self, distributed: bool = True):
        stats = self._sum_across_ranks(distributed)
        if float(stats[3]) > 0:
            mu = self.ema_rate
            for ema, total in zip((self.ema_num, self.ema_den, self.ema_r), stats[:3]):
                ema.mul_(1 - mu).add_(mu * total / stats[3])
            self.ema_steps += 1
        self._clear()

    @torch.no_grad()
    def freeze(self):
        if bool(self.frozen):
            return
        steps = float(self.ema_steps)
        if steps == 0:
            raise RuntimeError("TaperRMS.freeze() needs at least one committed warm-up statistic")
        correction = 1 - (1 - self.ema_rate) ** steps
        num, den, rr = self.ema_num / correction, self.ema_den / correction, self.ema_r / correction
        self.c.copy_(num / (den + 1e-30))
        self.s_tgt.copy_(rr)
        self.weight_tilde.copy_(self.weight)
        self.frozen.fill_(True)
        if not (torch.isfinite(self.c) and torch.isfinite(self.s_tgt)):
            raise FloatingPointError("the TaperNorm calibration is non-finite")


def taper_modules(model: nn.Module) -> list:
    return [m for m in model.modules() if isinstance(m, TaperRMS)]


def taper_gate(step: int, start: int, end: int) -> float:
    """Shared cosine gate: 1 up to ``start``, 0 from ``end`` on."""
    if step <= start:
        return 1.0
    if step >= end:
        return 0.0
    return 0.5 * (1 + math.cos(math.pi * (step - start) / (end - start)))


@torch.no_grad()
def taper_set_gate_(model: nn.Module, g: float):
    for m in taper_modules(model):
        m.gate.fill_(g)


def taper_anchor_loss(model: nn.Module) -> torch.Tensor | None:
    """Mean over tapered norms of their token-mean anchor term since the last call (then reset)."""
    terms = []
    for m in taper_modules(model):
        if m._anchor_sum is not None and m._anchor_count > 0:
            terms.append(m._anchor_sum / m._anchor_count)
        m._anchor_sum, m._anchor_count = None, 0.0
    return torch.stack(terms).mean() if terms else None


# ------------------------------------------------------------------------------------ spectral linear
def _kernel_ok(w: torch.Tensor) -> bool:
    return (w.is_cuda and w.dtype == torch.float32 and w.is_contiguous() and w.shape[1] % 4 == 0
            and not hasattr(w, "full_tensor"))


@torch.no_grad()
def power_iteration_step(w: torch.Tensor, u: torch.Tensor, v: torch.Tensor) -> None:
    """v <- normalize(W^T u), then u <- normalize(W v) in place; a vector whose new norm is not finite
    or at most SIGMA_FLOOR (e.g. W = 0) keeps its previous value.  u^T W v then estimates (from
    below) the largest singular value."""
    if _kernel_ok(w) and u.dtype == v.dtype == torch.float32:
        from ..ops._ext import lib
        lib().spectral_power_step(w, u, v, SIGMA_FLOOR)
        return
    wf = upcast(w)
    for vec, product in ((v, lambda: wf.t() @ u.to(wf.dtype)), (u, lambda: wf @ v.to(wf.dtype))):
        new = product()
        norm = new.norm()
        if torch.isfinite(norm) and norm > SIGMA_FLOOR:
            vec.copy_(new / norm)


class SpectralLinear(nn.Module):
    """``W_eff = gamma * W / sigma`` with ``sigma = |u^T W v|`` floored at SIGMA_FLOOR.  The forward
    never changes u or v (``spectral_step`` advances them once per optimizer step, before that step's
    forwards), so it is safe under gradient accumulation and recomputation."""

    def __init__(self, d_in: int, d_out: int, bias: bool = False):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(d_out, d_in))
        self.bias = nn.Parameter(torch.zeros(d_out)) if bias else None
        self.gamma = nn.Parameter(torch.ones(1))  # 1-D so that sharding layers can split it
        self.register_buffer("u", F.normalize(torch.randn(d_out), dim=0))
        self.register_buffer("v", F.normalize(torch.randn(d_in), dim=0))

    @property
    def in_features(self):
        return self.weight.shape[1]

    @property
    def out_features(self):
        return self.weight.shape[0]

    @torch.no_grad()
    def reset_gamma(self, iters: int = 50):
        """Start with W_eff equal to the freshly initialised W (gamma = sigma)."""
        if self.weight.is_meta:
            return
        for _ in range(iters):
            self._power_step()
        self.gamma.fill_(self.sigma_used().item())

    @torch.no_grad()
    def _power_step(self):
        w = self.weight.detach()
        full = getattr(w, "full_tensor", None)  # a sharded weight iterates on the full matrix
        power_iteration_step(full() if full is not None else w, self.u, self.v)

    def _sigma(self):
        w = upcast(self.weight)
        return self.u.to(w.dtype) @ w @ self.v.to(w.dtype)

    def sigma_used(self):
        return self._sigma().abs().clamp_min(SIGMA_FLOOR)

    def effective_weight(self):
        return (self.gamma * self.weight / self.sigma_used()).to(self.weight.dtype)

    def forward(self, x):
        # (gamma / sigma) W x on whichever side is smaller: the weight (d_in x d_out elements) or the
        # output (tokens x d_out elements); both are exact
        if x.numel() // x.shape[-1] > self.weight.shape[1]:
            return F.linear(x, self.effective_weight(), self.bias)
        y = F.linear(x, self.weight, None) * (self.gamma / self.sigma_used()).to(x.dtype)
        return y if self.bias is None else y + self.bias


@torch.no_grad()
def spectral_step(model: nn.Module):
    """Advance every SpectralLinear's power iteration once (once per optimizer step)."""
    for m in model.modules():
        if isinstance(m, SpectralLinear):
            m._power_step()


@torch.no_grad()
def freeze_spectral(model: nn.Module) -> int:
    """Replace every SpectralLinear by an nn.Linear holding its effective weight (the export path;
    logits are unchanged).  Returns how many were replaced."""
    swaps = [(parent, name, child) for parent in list(model.modules())
             for name, child in list(parent.named_children()) if isinstance(child, SpectralLinear)]
    for parent, name, child in swaps:
        w = child.effective_weight()
        plain = nn.Linear(w.shape[1], w.shape[0], bias=child.bias is not None, device=w.device, dtype=w.dtype)
        plain.weight.copy_(w)
        if child.bias is not None:
            plain.bias.copy_(child.bias)
        setattr(parent, name, plain)
    return len(swaps)


# ------------------------------------------------------------------------------------ helpers
_NORM_KINDS = {
    "rms": lambda d, cfg: RMSNorm(d, cfg.rms_eps),
    "group": lambda d, cfg: GroupRMSNorm(d, cfg.norm_groups, cfg.rms_eps),
    "lagged": lambda d, cfg: LaggedRMS(d, cfg.rms_eps, cfg.lagged_half_life_tokens),
    "taper": lambda d, cfg: TaperRMS(d, cfg.rms_eps, cfg.taper_ema_rate),
}


def make_norm(kind: str, d: int, cfg) -> nn.Module:
    if kind not in _NORM_KINDS:
        raise ValueError(f"unknown norm kind {kind!r}")
    return _NORM_KINDS[kind](d, cfg)


def dynamic_norms(model: nn.Module):
    return [(n, m) for n, m in model.named_modules() if isinstance(m, DynamicNorm)]


def lagged_modules(model: nn.Module):
    return [m for m in model.modules() if isinstance(m, LaggedRMS)]


def rms_jacobian(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    """Analytic Jacobian of RMSNorm at one vector: diag(g)/r - (g x) x^T / (d r^3)."""
    d = x.numel()
    r = math.sqrt(float(x @ x) / d + eps)
    return torch.diag(gamma) / r - torch.outer(gamma * x, x) / (d * r ** 3)
