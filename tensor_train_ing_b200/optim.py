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
same state layout (``momentum_buffer``).  On CUDA a matrix's update is five kernels of this
package: one pass for the clip scale, both lerps, the bf16 operand (already in the orientation the
iteration wants) and its sum of squares; one that divides by the bf16 Frobenius norm; the
Newton-Schulz steps, three tcgen05 GEMMs each whose epilogues fuse the affine combinations
(``B = b A + c A A``, ``X = a X + B X``); and one pass for decay, update and the bf16 weight copy
the next forward's GEMMs read.  ``FusedAdamW`` keeps torch AdamW's state layout and checkpoint
identity and runs its CUDA update as one multi-tensor kernel per group.  Both take the gradient
clip coefficient as a device scalar (``step(grad_scale=...)``), so the gradients are never
rescaled in a separate pass.
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


class _NSWorkspace:
    """Buffers of one Newton-Schulz shape (m <= n), reused across steps."""

    def __init__(self, m, n, device):
        self.x = torch.empty(m, n, device=device, dtype=torch.bfloat16)
        self.nxt = torch.empty_like(self.x)
        self.gram = torch.empty(m, m, device=device, dtype=torch.bfloat16)
        self.upd = torch.empty_like(self.gram)
        self.partial = torch.empty(1024, device=device, dtype=torch.float32)


def _newton_schulz_fused(x, steps, a, b, c, ws: _NSWorkspace | None = None):
    """Iterate on ``x`` (m <= n, bf16); returns the buffer holding the result (x or ws.nxt)."""
    from .ops._ext import lib
    C = lib()
    if ws is None:
        ws = _NSWorkspace(*x.shape, x.device)
    gram, upd, nxt = ws.gram, ws.upd, ws.nxt if ws.nxt.data_ptr() != x.data_ptr() else ws.x
    if _fused_ns_ok(x):
        for _ in range(steps):
            C.mm(x, x.t(), gram)                                  # A = X X^T
            C.mm(gram, gram, upd, gram, float(c), float(b))       # B = c A A + b A
            C.mm(upd, x, nxt, x, 1.0, float(a))                   # X = B X + a X
            x, nxt = nxt, x
        return x
    for _ in range(steps):  # shapes the GEMM kernel does not tile (tiny test models)
        g2 = x @ x.t()
        x = torch.addmm(x, torch.addmm(g2, g2, g2, beta=b, alpha=c), x, beta=a)
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

    accepts_grad_scale = True

    @torch.no_grad()
    def step(self, closure=None, grad_scale=None, caches=None, written=None):
        """``grad_scale``: optional device scalar the gradients are multiplied by (the clip
        coefficient); ``caches``: {id(param): bf16 [rows, cols] view} the update also writes,
        recorded in ``written``."""
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
                decay, alpha = 1 - lr * wd, -lr * muon_lr_ratio(group["adjust_lr_fn"], p.shape)
                if self._fused_ok(p, buf):
                    cache = caches.get(id(p)) if caches else None
                    self._fused_update(p, buf, group, decay, alpha, grad_scale, cache)
                    if cache is not None and written is not None:
                        written.add(id(p))
                    continue
                g = p.grad if grad_scale is None else p.grad * grad_scale
                buf.lerp_(g, 1 - mom)
                update = g.lerp(buf, mom) if group["nesterov"] else buf
                update = newton_schulz(update, group["ns_steps"], group["ns_coefficients"], group["eps"])
                p.mul_(decay)
                p.add_(update, alpha=alpha)
        return loss

    @staticmethod
    def _fused_ok(p, buf) -> bool:
        return (p.is_cuda and p.dtype == torch.float32 and p.grad.dtype == torch.float32 and p.is_contiguous()
                and p.grad.is_contiguous() and buf.is_contiguous())

    def _workspace(self, m, n, device) -> _NSWorkspace:
        spaces = self.__dict__.setdefault("_ns_spaces", {})
        key = (m, n, str(device))
        if key not in spaces:
            spaces[key] = _NSWorkspace(m, n, device)
        return spaces[key]

    def _fused_update(self, p, buf, group, decay, alpha, grad_scale, cache):
        from .ops._ext import lib
        C = lib()
        rows, cols = p.shape
        tall = rows > cols  # the iteration runs on the wide orientation
        ws = self._workspace(min(rows, cols), max(rows, cols), p.device)
        mom = group["momentum"]
        n_partial = C.muon_prepare(p.grad, buf, ws.x, ws.partial, float(1 - mom), float(mom),
                                   bool(group["nesterov"]), tall, grad_scale)
        C.muon_normalize(ws.x, ws.partial, n_partial, float(group["eps"]))
        a, b, c = group["ns_coefficients"]
        out = _newton_schulz_fused(ws.x, group["ns_steps"], a, b, c, ws)
        C.muon_apply(p, out.contiguous(), tall, float(decay), float(alpha), cache)


class FusedAdamW(torch.optim.AdamW):
    """torch AdamW's hyper-parameters, state layout (device ``step`` counters, ``exp_avg``,
    ``exp_avg_sq``) and checkpoint identity, with the CUDA update as this package's multi-tensor
    kernel: one launch per group covers every tensor, reads the clip coefficient from the device and
    can write bf16 copies of the updated weights.  Same arithmetic as torch's fused AdamW (decay
    ``p -= lr*wd*p``, moment updates, bias corrections from the per-tensor step counters)."""

    checkpoint_class = "torch.optim.adamw.AdamW"
    accepts_grad_scale = True

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, fused=True)
        self._tables: dict[int, tuple] = {}

    def load_state_dict(self, state_dict):
        """torch's load, then this optimizer's own layout: fused groups and every state tensor
        (the ``step`` counters included, which torch keeps on the host for a state saved by a
        non-fused AdamW) on its parameter's device, where the kernel reads them."""
        super().load_state_dict(state_dict)
        for group in self.param_groups:
            group.update(fused=True, foreach=None, capturable=False)
            for p in group["params"]:
                st = self.state.get(p)
                if st and "step" in st:
                    st["step"] = st["step"].to(device=p.device, dtype=torch.float32)
        self._tables = {}

    def _table(self, index, params, caches):
        rows, chunk = [], 16384
        first = 0
        for p in params:
            st = self.state[p]
            if any(st[k].device != p.device for k in ("step", "exp_avg", "exp_avg_sq")):
                raise ValueError("FusedAdamW state must live on its parameter's device")
            cache = caches.get(id(p)) if caches else None
            rows.append([p.data_ptr(), p.grad.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(),
                         st["step"].data_ptr(), cache.data_ptr() if cache is not None else 0, p.numel(), first])
            first += -(-p.numel() // chunk)
        key = tuple(tuple(r) for r in rows)
        held = self._tables.get(index)
        if held is None or held[0] != key:
            table = torch.tensor(rows, dtype=torch.int64).to(params[0].device, non_blocking=False)
            held = (key, table, first)
            self._tables[index] = held
        return held[1], held[2]

    @torch.no_grad()
    def step(self, closure=None, grad_scale=None, caches=None, written=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        from .ops._ext import lib
        for index, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            for p in params:
                if p.dtype != torch.float32 or not (p.is_contiguous() and p.grad.is_contiguous()):
                    raise ValueError("FusedAdamW updates contiguous fp32 parameters and gradients")
                st = self.state[p]
                if not st:
                    st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            table, chunks = self._table(index, params, caches)
            b1, b2 = group["betas"]
            lib().adamw_update(table, chunks, float(group["lr"]), float(b1), float(b2), float(group["eps"]),
                               float(group["weight_decay"]), grad_scale)
            if caches and written is not None:
                written.update(id(p) for p in params if id(p) in caches)
        return loss


def _adamw(groups, *, lr, betas):
    """AdamW over ``groups``: this package's kernel when every parameter is a CUDA tensor, torch's
    (its default implementation) otherwise."""
    params = [p for g in groups for p in g["params"]]
    if params and all(p.is_cuda for p in params):
        return FusedAdamW(groups, lr=lr, betas=betas)
    return torch.optim.AdamW(groups, lr=lr, betas=betas)


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
        # serial: only non-empty groups (the reference layout); sharded: every group on every rank
        self.adamw = _adamw(groups if only is not None else [g for g in groups if g["params"]], lr=aux_lr,
                            betas=betas)
        self.model = model
        # not calling Optimizer.__init__: the children own groups and state
        self.defaults = {}
        self._optimizer_step_pre_hooks, self._optimizer_step_post_hooks = {}, {}

    @property
    def accepts_grad_scale(self) -> bool:
        return getattr(self.adamw, "accepts_grad_scale", False)

    @property
    def param_groups(self):
        return self.muon.param_groups + self.adamw.param_groups

    @property
    def state(self):
        return {**self.muon.state, **self.adamw.state}

    @torch.no_grad()
    def step(self, closure=None, grad_scale=None):
        """Both children, then the bf16 operand caches whose every row the kernels rewrote are
        marked current (the forward's GEMMs use them without another conversion pass)."""
        if closure is not None:
            raise ValueError("MuonAdamW does not take a closure")
        if grad_scale is None:
            self.muon.step()
            self.adamw.step()
            return
        from .ops.weights import cache_views, mark_current
        caches, groups = cache_views(self.model)
        written: set[int] = set()
        self.muon.step(grad_scale=grad_scale, caches=caches, written=written)
        self.adamw.step(grad_scale=grad_scale, caches=caches, written=written)
        mark_current(groups, written)

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
        return _adamw(groups, lr=cfg.lr, betas=betas)
    if cfg.optimizer == "muon":
        if mult != 1.0:
            raise NotImplementedError("width/depth LR scaling is defined for AdamW only; Muon uses its own shape scaling")
        return MuonAdamW(model, lr=cfg.lr, aux_lr=cfg.aux_adamw_lr or cfg.lr, weight_decay=cfg.weight_decay_hidden,
                         betas=betas, momentum=cfg.muon_momentum, adjust_lr_fn=cfg.muon_adjust_lr, only=only)
    raise ValueError(f"unknown optimizer {cfg.optimizer!r}")
