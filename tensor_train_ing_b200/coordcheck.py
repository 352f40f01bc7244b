"""Coordinate checks across width (fixed depth and head dim) and across depth (fixed width)
(reference tnlm/coordcheck.py:20-104).

For each shape: RMS of every residual stream, attention and MLP branch output and the logits on a
fixed probe batch, at initialisation and after ``steps`` optimizer steps at a fixed LR, plus the RMS
of their change.  Log-log slopes against width (or depth) summarise the trend: near 0 means stable;
a positive slope of the change means the effective update grows with the dimension.  A diagnostic,
not a parameterisation proof.
"""
from __future__ import annotations

import math

import torch

from .config import ModelConfig, TrainConfig
from .models.model import TensorLM
from .optim import make_optimizer


def _rms(t) -> float:
    return float(t.detach().float().pow(2).mean().sqrt())


@torch.no_grad()
def _probe(model, idx) -> dict:
    stats, hooks = {}, []
    for i, blk in enumerate(model.blocks):
        hooks.append(blk.register_forward_hook(lambda m, a, o, i=i: stats.__setitem__(f"resid{i}", o)))
        hooks.append(blk.attn.register_forward_hook(lambda m, a, o, i=i: stats.__setitem__(f"attn{i}", o)))
        hooks.append(blk.mlp.register_forward_hook(lambda m, a, o, i=i: stats.__setitem__(f"mlp{i}", o)))
    model._force_reference = True  # module hooks need the module-level path
    try:
        stats["logits"] = model(idx)
    finally:
        model._force_reference = False
        for h in hooks:
            h.remove()
    return {k: v.detach().float().clone() for k, v in stats.items()}


def _batch(g, batch, context, vocab, task):
    x = torch.randint(0, vocab, (batch, context), generator=g)
    if task == "repeat":  # second half copies the first: a learnable signal
        x[:, context // 2:] = x[:, : context - context // 2]
    return x


def _slopes(xs, rows, keys) -> dict:
    lx = [math.log(x) for x in xs]
    out = {}
    for key in keys:
        for f in ("init", "delta"):
            ly = [math.log(max(rows[x][key][f], 1e-30)) for x in xs]
            mx, my = sum(lx) / len(lx), sum(ly) / len(ly)
            out[f"{key}.{f}"] = sum((a - mx) * (b - my) for a, b in zip(lx, ly)) / sum((a - mx) ** 2 for a in lx)
    return out


def run(widths=(256, 512, 1024), *, layers=4, head_dim=64, steps=3, lr=4.5e-4, optimizer="adamw", batch=8,
        context=256, vocab=8192, device=None, seed=0, task="random", train_kw=None, **model_kw) -> dict:
    """Width check.  ``train_kw``: extra TrainConfig fields (e.g. ``{"muon_adjust_lr": "spectral_unclamped"}``)."""
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    rows = {}
    for w in widths:
        torch.manual_seed(seed)
        poly = model_kw.get("attention", "signed_product") != "softmax"
        d_mlp = model_kw.get("d_mlp", int(round((4 * w - (2 * w / 3 if poly else 0)) / 64) * 64))
        cfg = ModelConfig(layers=layers, d_model=w, heads=w // head_dim, d_key=head_dim, d_value=head_dim,
                          d_mlp=d_mlp, vocab_size=vocab, padded_vocab=vocab,
                          **{k: v for k, v in model_kw.items() if k != "d_mlp"})
        m = TensorLM(cfg).to(device).train()
        opt = make_optimizer(m, TrainConfig(optimizer=optimizer, lr=lr, **(train_kw or {})))
        g = torch.Generator().manual_seed(seed + 1)
        probe = _batch(g, batch, context, vocab, task).to(device)
        init = _probe(m, probe)
        for _ in range(steps):
            idx = _batch(g, batch, context, vocab, task).to(device)
            _, loss = m(idx, targets=idx.roll(-1, 1))
            loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
        after = _probe(m, probe)
        rows[w] = {k: {"init": _rms(init[k]), "after": _rms(after[k]), "delta": _rms(after[k] - init[k])} for k in init}
        del m, opt
    slopes = _slopes(list(widths), rows, rows[widths[0]]) if len(widths) > 1 else {}
    return {"widths": list(widths), "layers": layers, "head_dim": head_dim, "optimizer": optimizer, "lr": lr,
            "task": task, "steps": steps, "rows": rows, "loglog_slopes": slopes}


def run_depth(depths=(2, 4, 8, 16), *, width=512, **kw) -> dict:
    """Depth check: first/last block quantities and logits, slopes against depth."""
    rows = {}
    for L in depths:
        r = run(widths=(width,), layers=L, **kw)["rows"][width]
        rows[L] = {"resid_first": r["resid0"], "resid_last": r[f"resid{L - 1}"], "attn_last": r[f"attn{L - 1}"],
                   "mlp_last": r[f"mlp{L - 1}"], "logits": r["logits"]}
    return {"depths": list(depths), "width": width, "rows": rows,
            "loglog_slopes": _slopes(list(depths), rows, rows[depths[0]]) if len(depths) > 1 else {}}


if __name__ == "__main__":
    import json
    import sys
    r = run(optimizer=sys.argv[1] if len(sys.argv) > 1 else "adamw",
            lr=float(sys.argv[2]) if len(sys.argv) > 2 else 4.5e-4)
    print(json.dumps({k: round(v, 2) for k, v in r["loglog_slopes"].items()}))
