"""Coordinate checks: how activation and update sizes scale with width (fixed depth and head
dimension) or with depth (fixed width).

For each shape a model is built from the same seed, a fixed probe batch is run at initialisation and
after ``steps`` optimizer updates at one learning rate, and the RMS of every residual stream, every
attention and MLP branch output and the logits is recorded, with the RMS of their change.  A
least-squares slope of log RMS against log width (or depth) summarises each trend: near 0 means the
quantity is stable across shapes; a positive slope of the change means the effective update grows
with the dimension, so a learning rate tuned at one size will not transfer unchanged.  A diagnostic,
not a derivation of a parameterisation.  Same measurements and report as the reference's check
(tnlm/coordcheck.py:20-104).
"""
from __future__ import annotations

import math
from contextlib import contextmanager

import torch

from .config import ModelConfig, TrainConfig
from .models.model import TensorLM
from .optim import make_optimizer


def _rms(t) -> float:
    return float(t.detach().float().pow(2).mean().sqrt())


def loglog_slope(xs, ys) -> float:
    """Least-squares slope of log y against log x (y floored at 1e-30)."""
    lx = [math.log(x) for x in xs]
    ly = [math.log(max(y, 1e-30)) for y in ys]
    mx, my = sum(lx) / len(lx), sum(ly) / len(ly)
    return sum((a - mx) * (b - my) for a, b in zip(lx, ly)) / sum((a - mx) ** 2 for a in lx)


@contextmanager
def _captured(model):
    """Record each block's output (resid<i>) and its attention and MLP branch outputs while the
    model runs its module-level path (the fused path does not call the submodules' forwards)."""
    seen, handles = {}, []

    def keep(name):
        return lambda _m, _inputs, out: seen.__setitem__(name, out.detach().float().clone())
    for i, blk in enumerate(model.blocks):
        handles += [blk.register_forward_hook(keep(f"resid{i}")), blk.attn.register_forward_hook(keep(f"attn{i}")),
                    blk.mlp.register_forward_hook(keep(f"mlp{i}"))]
    forced = getattr(model, "_force_reference", False)
    model._force_reference = True
    try:
        yield seen
    finally:
        model._force_reference = forced
        for h in handles:
            h.remove()


@torch.no_grad()
def _probe(model, idx) -> dict:
    with _captured(model) as seen:
        seen["logits"] = model(idx).detach().float().clone()
    return dict(seen)


def _token_batch(gen, batch, context, vocab, task):
    x = torch.randint(0, vocab, (batch, context), generator=gen)
    if task == "repeat":  # the second half repeats the first: a signal the model can learn
        x[:, context // 2:] = x[:, : context - context // 2]
    return x


def _default_d_mlp(width: int, attention: str) -> int:
    """The check's default MLP width: 4 w, less 2 w / 3 with polynomial attention (whose second
    query/key pair adds parameters), rounded to a multiple of 64."""
    spent = 2 * width / 3 if attention != "softmax" else 0
    return int(round((4 * width - spent) / 64) * 64)


def _measure(cfg: ModelConfig, *, steps, lr, optimizer, batch, context, vocab, device, seed, task, train_kw) -> dict:
    torch.manual_seed(seed)
    model = TensorLM(cfg).to(device).train()
    opt = make_optimizer(model, TrainConfig(optimizer=optimizer, lr=lr, **(train_kw or {})))
    gen = torch.Generator().manual_seed(seed + 1)
    probe = _token_batch(gen, batch, context, vocab, task).to(device)
    before = _probe(model, probe)
    for _ in range(steps):
        idx = _token_batch(gen, batch, context, vocab, task).to(device)
        _, loss = model(idx, targets=idx.roll(-1, 1))
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
    after = _probe(model, probe)
    return {k: {"init": _rms(before[k]), "after": _rms(after[k]), "delta": _rms(after[k] - before[k])} for k in before}


def _slopes(dims, rows) -> dict:
    if len(dims) < 2:
        return {}
    return {f"{key}.{field}": loglog_slope(dims, [rows[x][key][field] for x in dims])
            for key in rows[dims[0]] for field in ("init", "delta")}


def run(widths=(256, 512, 1024), *, layers=4, head_dim=64, steps=3, lr=4.5e-4, optimizer="adamw", batch=8,
        context=256, vocab=8192, device=None, seed=0, task="random", train_kw=None, **model_kw) -> dict:
    """Width check.  ``train_kw``: extra TrainConfig fields (e.g. ``{"muon_adjust_lr": "spectral_unclamped"}``);
    ``model_kw``: extra ModelConfig fields (``d_mlp`` overrides the default width)."""
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    extra = {k: v for k, v in model_kw.items() if k != "d_mlp"}
    rows = {}
    for w in widths:
        d_mlp = model_kw.get("d_mlp", _default_d_mlp(w, model_kw.get("attention", "signed_product")))
        cfg = ModelConfig(layers=layers, d_model=w, heads=w // head_dim, d_key=head_dim, d_value=head_dim,
                          d_mlp=d_mlp, vocab_size=vocab, padded_vocab=vocab, **extra)
        rows[w] = _measure(cfg, steps=steps, lr=lr, optimizer=optimizer, batch=batch, context=context, vocab=vocab,
                           device=device, seed=seed, task=task, train_kw=train_kw)
    return {"widths": list(widths), "layers": layers, "head_dim": head_dim, "optimizer": optimizer, "lr": lr,
            "task": task, "steps": steps, "rows": rows, "loglog_slopes": _slopes(list(widths), rows)}


def run_depth(depths=(2, 4, 8, 16), *, width=512, **kw) -> dict:
    """Depth check at one width: the first and last block's stream, the last block's branches and the
    logits, with slopes against depth."""
    rows = {}
    for L in depths:
        r = run(widths=(width,), layers=L, **kw)["rows"][width]
        last = L - 1
        rows[L] = {"resid_first": r["resid0"], "resid_last": r[f"resid{last}"], "attn_last": r[f"attn{last}"],
                   "mlp_last": r[f"mlp{last}"], "logits": r["logits"]}
    return {"depths": list(depths), "width": width, "rows": rows, "loglog_slopes": _slopes(list(depths), rows)}


if __name__ == "__main__":
    import json
    import sys
    report = run(optimizer=sys.argv[1] if len(sys.argv) > 1 else "adamw",
                 lr=float(sys.argv[2]) if len(sys.argv) > 2 else 4.5e-4)
    print(json.dumps({k: round(v, 2) for k, v in report["loglog_slopes"].items()}))
