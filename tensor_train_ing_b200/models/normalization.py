"""Normalisation modules and the spectral (sigma-reparameterised) linear map.

Module, parameter and buffer names follow the reference (tnlm/normalization.py:15-381) so that
its checkpoints load into this framework:

  RMSNorm / GroupRMSNorm   weight                                         class "N"
  LaggedRMS                weight, mean_sq, calibrated                    class "P"
  TaperRMS                 weight, weight_tilde, gate, c, s_tgt,          "N" until frozen at gate 0
                           ema_num, ema_den, ema_r, ema_steps, frozen
  SpectralLinear           weight, [bias], gamma, u, v

All reductions run in at least fp32.  These modules define the math; on CUDA the model's fused
path calls the sm_100a norm kernels (``tensor_train_ing_b200.ops.norm``) for RMSNorm and the
lagged/taper divisions instead of these forwards.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

SIGMA_FLOOR = 1e-12


def upcast(x: torch.Tensor) -> torch.Tensor:
    """Reduction dtype: fp32, or fp64 when the input already is fp64 (oracle tests)."""
    return x.to(torch.promote_types(x.dtype, torch.float32))


class DynamicNorm(nn.Module):
    """Input-dependent normaliser ``x / r(x) * weight`` with analysis hooks on the denominator.

    ``denom_mode``: None (training), "record" (store r), "clamp" (reuse the stored r) or "const"
    (use ``denom_const``).  Analysis modes are rejected while the module is in training mode.
    """

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

    def forward(self, x):
        if self.denom_mode is not None and self.training:
            raise RuntimeError("denom_mode is analysis-only; reset it before training")
        r = self.denom(x)
        mode = self.denom_mode
        if mode == "record":
            self.denom_saved = r.detach()
        elif mode == "clamp":
            r = self.denom_saved.to(r.dtype)
        elif mode == "const":
            r = self.denom_const.to(device=r.device, dtype=r.dtype).expand_as(r)
        return (upcast(x) / r * upcast(self.weight)).to(x.dtype)


class RMSNorm(DynamicNorm):
    def denom(self, x):
        xf = upcast(x)
        return (xf.square().mean(dim=-1, keepdim=True) + self.eps).sqrt()


class GroupRMSNorm(DynamicNorm):
    """RMS over ``groups`` contiguous feature groups (a per-token, per-group denominator)."""

    def __init__(self, d: int, groups: int = 4, eps: float = 1e-6):
        super().__init__(d, eps)
        if d % groups:
            raise ValueError("d must be divisible by groups")
        self.groups = groups

    def denom(self, x):
        xg = upcast(x).unflatten(-1, (self.groups, -1))
        r = (xg.square().mean(dim=-1, keepdim=True) + self.eps).sqrt()
        return r.expand_as(xg).flatten(-2)


class LaggedRMS(nn.Module):
    """Divide by a detached, lagged scalar RMS: ``x / sqrt(mean_sq + eps) * weight``.

    The current batch never influences its own output.  With ``collecting`` on, forward also
    accumulates count-weighted sums of the per-token mean square (padding excluded through
    ``set_valid_mask``); ``commit`` folds them into ``mean_sq`` with a token half-life EMA, once
    per optimizer step (summed across data-parallel ranks first so the buffer stays replicated).
    """

    op_class = "P"

    def __init__(self, d: int, eps: float = 1e-6, half_life_tokens: float = 1e6):
        super().__init__()
        self.eps = eps
        self.half_life_tokens = half_life_tokens
        self.weight = nn.Parameter(torch.ones(d))
        self.register_buffer("mean_sq", torch.ones((), dtype=torch.float64))
        self.register_buffer("calibrated", torch.zeros((), dtype=torch.bool))
        self.register_buffer("acc_sum", torch.zeros((), dtype=torch.float64), persistent=False)
        self.register_buffer("acc_count", torch.zeros((), dtype=torch.float64), persistent=False)
        self.collecting = False
        self._valid: torch.Tensor | None = None

    def set_valid_mask(self, valid: torch.Tensor | None):
        self._valid = valid

    def denom(self, x):
        # sqrt in fp64 first so very large statistics still fit the fp32 divisor
        return (self.mean_sq + self.eps).sqrt().to(torch.promote_types(x.dtype, torch.float32))

    @torch.no_grad()
    def observe(self, x: torch.Tensor):
        per_token = x.detach().double().square().mean(dim=-1)
        if self._valid is not None:
            per_token = per_token * self._valid
            count = self._valid.sum().double()
        else:
            count = torch.tensor(float(per_token.numel()), device=per_token.device, dtype=torch.float64)
        self.acc_sum += per_token.sum()
        self.acc_count += count

    def forward(self, x):
        if self.collecting:
            self.observe(x)
        return (upcast(x) / self.denom(x) * upcast(self.weight)).to(x.dtype)

    @torch.no_grad()
    def commit(self, distributed: bool = True) -> float:
        if distributed and torch.distributed.is_available() and torch.distributed.is_initialized():
            stats = torch.stack([self.acc_sum, self.acc_count])
            torch.distributed.all_reduce(stats)
            self.acc_sum.copy_(stats[0])
            self.acc_count.copy_(stats[1])
        n = float(self.acc_count)
        if n == 0:
            return float(self.mean_sq)
        batch_ms = self.acc_sum / self.acc_count
        if bool(self.calibrated):
            keep = 0.5 ** (n / self.half_life_tokens)
            self.mean_sq.mul_(keep).add_((1 - keep) * batch_ms)
        else:
            self.mean_sq.copy_(batch_ms)
            self.calibrated.fill_(True)
        self.acc_sum.zero_()
        self.acc_count.zero_()
        if not torch.isfinite(self.mean_sq):
            raise FloatingPointError("non-finite lagged RMS statistic")
        return float(self.mean_sq)


class TaperRMS(nn.Module):
    """TaperNorm, RMS form: ``g * x/r(x) * weight + (1 - g) * c * x * weight_tilde``.

    g = 1 is RMSNorm; g = 0 is a fixed diagonal map (class "P").  Lifecycle driven by the trainer:
    warm-up statistics (``collecting``/``commit``), ``freeze`` (c = E[|xw|^2/r]/E[|xw|^2],
    s_tgt = E[r], weight_tilde <- weight), then a shared cosine gate 1 -> 0; while frozen and
    training, forward accumulates the differentiable anchor (r - s_tgt)^2 read by
    ``taper_anchor_loss``.
    """

    def __init__(self, d: int, eps: float = 1e-6, ema_rate: float = 0.01):
        super().__init__()
        self.eps = eps
        self.ema_rate = ema_rate
        self.weight = nn.Parameter(torch.ones(d))
        self.weight_tilde = nn.Parameter(torch.ones(d))
        for name, init in (("gate", 1.0), ("c", 1.0), ("s_tgt", 1.0), ("ema_num", 0.0), ("ema_den", 0.0),
                           ("ema_r", 0.0), ("ema_steps", 0.0)):
            self.register_buffer(name, torch.tensor(init, dtype=torch.float64))
        self.register_buffer("frozen", torch.zeros((), dtype=torch.bool))
        for name in ("acc_num", "acc_den", "acc_r", "acc_count"):
            self.register_buffer(name, torch.zeros((), dtype=torch.float64), persistent=False)
        self.collecting = False
        self._valid: torch.Tensor | None = None
        self._anchor_sum: torch.Tensor | None = None
        self._anchor_count = 0.0

    @property
    def op_class(self):
        return "P" if bool(self.frozen) and float(self.gate) == 0.0 else "N"

    def set_valid_mask(self, valid: torch.Tensor | None):
        self._valid = valid

    def forward(self, x):
        xf = upcast(x)
        g = float(self.gate)
        frozen = bool(self.frozen)
        r = None
        if g > 0 or self.collecting or (self.training and frozen):
            r = (xf.square().mean(dim=-1, keepdim=True) + self.eps).sqrt()
        if self.collecting and not frozen:
            with torch.no_grad():
                sq = (xf.detach() * upcast(self.weight.detach())).double().square().sum(dim=-1)
                rr = r.detach().double().squeeze(-1)
                w = self._valid.double() if self._valid is not None else torch.ones_like(rr)
                self.acc_num += (sq / rr * w).sum()
                self.acc_den += (sq * w).sum()
                self.acc_r += (rr * w).sum()
                self.acc_count += w.sum()
        if self.training and frozen:
            dev = (r.squeeze(-1) - self.s_tgt.to(r.dtype)).square()
            if self._valid is not None:
                dev = dev * self._valid
                n = float(self._valid.sum())
            else:
                n = float(dev.numel())
            total = dev.sum()
            self._anchor_sum = total if self._anchor_sum is None else self._anchor_sum + total
            self._anchor_count += n
        linear = float(self.c) * xf * upcast(self.weight_tilde)
        if g == 0.0:
            return linear.to(x.dtype)
        normed = xf / r * upcast(self.weight)
        if g == 1.0:
            return normed.to(x.dtype)
        return (g * normed + (1 - g) * linear).to(x.dtype)

    @torch.no_grad()
    def commit(self, distributed: bool = True):
        stats = torch.stack([self.acc_num, self.acc_den, self.acc_r, self.acc_count])
        if distributed and torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.all_reduce(stats)
        if float(stats[3]) > 0:
            mu = self.ema_rate
            for ema, total in ((self.ema_num, stats[0]), (self.ema_den, stats[1]), (self.ema_r, stats[2])):
                ema.mul_(1 - mu).add_(mu * total / stats[3])
            self.ema_steps += 1
        for acc in (self.acc_num, self.acc_den, self.acc_r, self.acc_count):
            acc.zero_()

    @torch.no_grad()
    def freeze(self):
        if bool(self.frozen):
            return
        steps = float(self.ema_steps)
        if steps == 0:
            raise RuntimeError("TaperRMS.freeze() before any committed warmup statistics")
        correction = 1 - (1 - self.ema_rate) ** steps
        num, den, rr = self.ema_num / correction, self.ema_den / correction, self.ema_r / correction
        self.c.copy_(num / (den + 1e-30))
        self.s_tgt.copy_(rr)
        self.weight_tilde.copy_(self.weight)
        self.frozen.fill_(True)
        if not (torch.isfinite(self.c) and torch.isfinite(self.s_tgt)):
            raise FloatingPointError("non-finite TaperNorm calibration")


def taper_modules(model: nn.Module) -> list:
    return [m for m in model.modules() if isinstance(m, TaperRMS)]


def taper_gate(step: int, start: int, end: int) -> float:
    """Cosine gate: 1 up to ``start``, 0 from ``end`` on."""
    if step <= start:
        return 1.0
    if step >= end:
        return 0.0
    return 0.5 * (1.0 + math.cos(math.pi * (step - start) / (end - start)))


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


class SpectralLinear(nn.Module):
    """sigma-reparameterised linear map: ``W_eff = gamma * W / sigma``, sigma = |u^T W v|.

    u and v are power-iteration buffers that forward never mutates; ``spectral_step`` advances
    them once per optimizer step.  ``effective_weight`` is the exported matrix.
    """

    def __init__(self, d_in: int, d_out: int, bias: bool = False):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(d_out, d_in))
        self.bias = nn.Parameter(torch.zeros(d_out)) if bias else None
        self.gamma = nn.Parameter(torch.ones(1))
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
        """Make W_eff equal the freshly initialised W (gamma = sigma)."""
        if self.weight.is_meta:
            return
        for _ in range(iters):
            self._power_step()
        self.gamma.fill_(self.sigma_used().item())

    def _full_weight(self):
        w = self.weight.detach()
        full = getattr(w, "full_tensor", None)  # DTensor shards: iterate on the full matrix
        return upcast(full() if full is not None else w)

    @torch.no_grad()
    def _power_step(self):
        """One power-iteration step; a vector that collapses (e.g. W = 0) keeps its old value."""
        w = self._full_weight()
        v_new = w.t() @ self.u.to(w.dtype)
        n = v_new.norm()
        if torch.isfinite(n) and n > SIGMA_FLOOR:
            self.v.copy_(v_new / n)
        u_new = w @ self.v.to(w.dtype)
        n = u_new.norm()
        if torch.isfinite(n) and n > SIGMA_FLOOR:
            self.u.copy_(u_new / n)

    def _sigma(self):
        w = upcast(self.weight)
        return self.u.to(w.dtype) @ w @ self.v.to(w.dtype)

    def sigma_used(self):
        return self._sigma().abs().clamp_min(SIGMA_FLOOR)

    def effective_weight(self):
        return (self.gamma * self.weight / self.sigma_used()).to(self.weight.dtype)

    def forward(self, x):
        # Scale whichever side is smaller: the weight (d_in*d_out) or the output (tokens*d_out).
        if x.numel() // x.shape[-1] > self.weight.shape[1]:
            return F.linear(x, self.effective_weight(), self.bias)
        y = F.linear(x, self.weight, None) * (self.gamma / self.sigma_used()).to(x.dtype)
        return y if self.bias is None else y + self.bias


def make_norm(kind: str, d: int, cfg) -> nn.Module:
    if kind == "rms":
        return RMSNorm(d, cfg.rms_eps)
    if kind == "group":
        return GroupRMSNorm(d, cfg.norm_groups, cfg.rms_eps)
    if kind == "lagged":
        return LaggedRMS(d, cfg.rms_eps, cfg.lagged_half_life_tokens)
    if kind == "taper":
        return TaperRMS(d, cfg.rms_eps, cfg.taper_ema_rate)
    raise ValueError(f"unknown norm kind {kind!r}")


@torch.no_grad()
def spectral_step(model: nn.Module):
    """Advance every SpectralLinear's power iteration once (call once per optimizer step)."""
    for m in model.modules():
        if isinstance(m, SpectralLinear):
            m._power_step()


@torch.no_grad()
def freeze_spectral(model: nn.Module) -> int:
    """Swap every SpectralLinear for an nn.Linear holding its effective weight; returns the count."""
    replaced = 0
    for parent in list(model.modules()):
        for name, child in list(parent.named_children()):
            if not isinstance(child, SpectralLinear):
                continue
            w = child.effective_weight()
            plain = nn.Linear(w.shape[1], w.shape[0], bias=child.bias is not None, device=w.device, dtype=w.dtype)
            plain.weight.copy_(w)
            if child.bias is not None:
                plain.bias.copy_(child.bias)
            setattr(parent, name, plain)
            replaced += 1
    return replaced


def dynamic_norms(model: nn.Module):
    return [(n, m) for n, m in model.named_modules() if isinstance(m, DynamicNorm)]


def lagged_modules(model: nn.Module):
    return [m for m in model.modules() if isinstance(m, LaggedRMS)]


def rms_jacobian(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    """Analytic Jacobian of RMSNorm at one vector: diag(g)/r - (g*x) x^T / (d r^3)."""
    d = x.numel()
    r = math.sqrt(float(x @ x) / d + eps)
    return torch.diag(gamma) / r - torch.outer(gamma * x, x) / (d * r ** 3)
