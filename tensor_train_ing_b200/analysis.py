"""Interpretability diagnostics of a trained TensorLM (reference tnlm/analysis.py:29-596).

``analyze(model, batches, out_dir)`` writes a JSON report with:
  1. local tensors: the bilinear MLP's symmetric coefficient tensor restricted to a random subspace
     (reconstructs the module exactly) and the gain-folded form on probe activations;
  2. read/write graph: cosine overlaps of upstream write directions with downstream read vectors;
  3. normalizer sensitivity: per-site denominators, analytic vs autograd JVPs, radial/direct ratio;
  4. ablation decomposition: branch removal with live vs clamped denominators;
  5. fixed denominators: calibrated constant denominators vs live ones;
  6. low-rank structure of MLP quadratic forms and per-head QK bilinear forms;
  7. stability statistics (max |S|, |S1 S2|, bilinear-product tails) shared with QK-clip.

All diagnostics run on the reference (PyTorch) path of the model, where norm modules expose their
denominators and forward hooks see every sublayer; the fused kernels are bypassed inside
``reference_path(model)``.
"""
from __future__ import annotations

import hashlib
import json
import math
from contextlib import contextmanager
from pathlib import Path

import torch
import torch.nn as nn
import torch.nn.functional as F

from .models.attention import apply_rope, doc_positions, rope_tables, visible_mask
from .models.normalization import (DynamicNorm, GroupRMSNorm, LaggedRMS, RMSNorm, SpectralLinear, TaperRMS,
                                   dynamic_norms, upcast)

QUANTILES = (0.01, 0.05, 0.5, 0.95, 0.99)
POS_BUCKETS = ((0, 16), (16, 64), (64, 256), (256, 1 << 30))


@contextmanager
def reference_path(model):
    """Run the model through its PyTorch reference path (hooks and denominator modes visible)."""
    prev = getattr(model, "_force_reference", False)
    model._force_reference = True
    try:
        yield model
    finally:
        model._force_reference = prev


def eff(lin: nn.Module) -> torch.Tensor:
    return upcast((lin.effective_weight() if isinstance(lin, SpectralLinear) else lin.weight).detach())


def gain(norm: nn.Module, d: int, device) -> torch.Tensor:
    """The fixed per-feature map of a norm site that folds into the adjacent linear maps."""
    if isinstance(norm, TaperRMS):
        g = float(norm.gate)
        if g == 1.0:
            return upcast(norm.weight.detach())
        if g == 0.0 and bool(norm.frozen):
            return float(norm.c) * upcast(norm.weight_tilde.detach())
        raise ValueError(f"TaperRMS at gate {g} (frozen={bool(norm.frozen)}) has no fixed foldable map")
    w = getattr(norm, "weight", None)
    if w is None:
        return torch.ones(d, device=device)
    out = upcast(w.detach())
    if isinstance(norm, LaggedRMS):
        out = out / torch.sqrt(norm.mean_sq.detach().to(out.dtype) + norm.eps)
    return out


def norm_scope(norm: nn.Module) -> str:
    if isinstance(norm, GroupRMSNorm):
        return f"per-token RMS over {norm.groups} contiguous feature groups"
    if isinstance(norm, RMSNorm):
        return "per-token RMS over all features"
    if isinstance(norm, LaggedRMS):
        return "frozen scalar (constant at checkpoint)"
    if isinstance(norm, TaperRMS):
        if bool(norm.frozen) and float(norm.gate) == 0.0:
            return "fixed diagonal scale c*gamma_tilde (tapered; constant at checkpoint)"
        return f"per-token RMS, taper gate {float(norm.gate):g}"
    return "none"


def _quantiles(x: torch.Tensor) -> dict:
    x = upcast(x.flatten())
    if x.numel() == 0:
        return {}
    if x.numel() > 1_000_000:
        x = x[torch.randperm(x.numel(), device=x.device)[:1_000_000]]
    qs = torch.quantile(x, torch.tensor(QUANTILES, device=x.device, dtype=x.dtype))
    return {**{f"q{int(p * 100):02d}": float(v) for p, v in zip(QUANTILES, qs)}, "mean": float(x.mean())}


@contextmanager
def _restore_modes(model):
    try:
        yield
    finally:
        for _, m in dynamic_norms(model):
            m.denom_mode, m.denom_saved, m.denom_const = None, None, None
        for blk in model.blocks:
            blk.ablate = frozenset()


def _set_mode(model, mode):
    for _, m in dynamic_norms(model):
        m.denom_mode = mode


def _token_losses(model, idx, doc, tgt):
    logits = upcast(model(idx, doc))
    loss = F.cross_entropy(logits.flatten(0, 1), tgt.flatten(), ignore_index=-100, reduction="none")
    return logits, loss.view_as(tgt)


def _doc_keys(doc, tgt):
    valid = tgt != -100
    key = torch.arange(doc.shape[0], device=doc.device)[:, None] * (doc.max() + 2) + doc.clamp_min(0)
    return key[valid], valid


def _paired_doc_stats(diffs, keys) -> dict:
    """Mean of per-document mean CE differences and its standard error across documents."""
    per_doc = []
    for d, k in zip(diffs, keys):
        uk, inv = torch.unique(k, return_inverse=True)
        s = torch.zeros(len(uk), device=d.device, dtype=torch.float64).index_add_(0, inv, d.double())
        c = torch.zeros(len(uk), device=d.device, dtype=torch.float64).index_add_(0, inv, torch.ones_like(d, dtype=torch.float64))
        per_doc.append(s / c)
    v = torch.cat(per_doc)
    n = v.numel()
    return {"mean": float(v.mean()), "doc_se": float(v.std(unbiased=True) / math.sqrt(n)) if n > 1 else float("nan"),
            "documents": n}


# ---------------------------------------------------------------------------------- 1. local tensors
@torch.no_grad()
def mlp_local_tensor(blk, basis: torch.Tensor, fold_gain: bool = True):
    """Symmetrised coefficient tensor (d_out, k[+1], k[+1]) of the MLP on span(basis)."""
    m = blk.mlp
    L, R, D = eff(m.l), eff(m.r), eff(m.d)
    if fold_gain:
        g = gain(blk.mlp_in, L.shape[1], L.device)
        L, R = L * g, R * g
    basis = basis.to(L.dtype)
    LU, RU = L @ basis, R @ basis
    bL, bR, bD = (getattr(lin, "bias", None) for lin in (m.l, m.r, m.d))
    if bL is not None:
        LU = torch.cat([LU, upcast(bL.detach())[:, None]], 1)
        RU = torch.cat([RU, upcast(bR.detach())[:, None]], 1)
        e = torch.zeros(1, LU.shape[1], device=LU.device, dtype=LU.dtype)
        e[0, -1] = 1
        LU, RU = torch.cat([LU, e]), torch.cat([RU, e])
        D = torch.cat([D, upcast(bD.detach())[:, None]], 1)
    T = torch.einsum("oh,ha,hb->oab", D, LU, RU)
    return 0.5 * (T + T.transpose(1, 2))


@torch.no_grad()
def local_tensor_check(model, hidden, k: int = 8, n: int = 16) -> dict:
    rows = []
    gen = torch.Generator(device="cpu").manual_seed(0)
    for i, blk in enumerate(model.blocks):
        if blk.mlp.kind == "swiglu":
            rows.append({"layer": i, "skipped": "SwiGLU is class G"})
            continue
        d = model.cfg.d_model
        dev = blk.mlp.l.weight.device
        dt = upcast(blk.mlp.l.weight).dtype
        U = torch.linalg.qr(torch.randn(d, k, generator=gen, dtype=torch.float64)).Q.to(device=dev, dtype=dt)
        z = torch.randn(n, k, generator=gen, dtype=torch.float64).to(device=dev, dtype=dt)
        T = mlp_local_tensor(blk, U, fold_gain=False)
        za = torch.cat([z, torch.ones(n, 1, device=dev, dtype=dt)], 1) if T.shape[1] > k else z
        rec = torch.einsum("oab,na,nb->no", T, za, za)
        ref = upcast(blk.mlp(z @ U.T))
        row = {"layer": i, "subspace_rank": k,
               "rel_err_restricted_tensor": float((rec - ref).norm() / ref.norm().clamp_min(1e-30))}
        norm = blk.mlp_in
        if type(norm) is RMSNorm and blk.mlp.kind == "bilinear":
            x = upcast(hidden[i][1].reshape(-1, d)[:256])
            g = gain(norm, d, dev)
            r = torch.sqrt(x.square().mean(-1, keepdim=True) + norm.eps)
            L, R, D = eff(blk.mlp.l), eff(blk.mlp.r), eff(blk.mlp.d)
            folded = (((x * g) @ L.T) * ((x * g) @ R.T)) @ D.T / r ** 2
            live = upcast(blk.mlp(norm(x)))
            row["rel_err_gain_folded_on_probe"] = float((folded - live).norm() / live.norm().clamp_min(1e-30))
        rows.append(row)
    return {"per_layer": rows, "max_rel_err": max((r.get("rel_err_restricted_tensor", 0) for r in rows), default=0.0)}


# ---------------------------------------------------------------------------------- 2. read/write graph
def _writers(model):
    for i, blk in enumerate(model.blocks):
        for comp, lin, onorm in (("attn", blk.attn.o, blk.attn_out), ("mlp", blk.mlp.d, blk.mlp_out)):
            W = eff(lin)
            if isinstance(onorm, DynamicNorm):
                W = W * gain(onorm, W.shape[0], W.device)[:, None]
            yield (i, comp), W, norm_scope(onorm)


def _readers(model, after_layer, after_comp, layer_window=None):
    dev = model.unembed.weight.device
    for j, blk in enumerate(model.blocks):
        if layer_window is not None and j > after_layer + layer_window:
            break
        a = blk.attn
        if j > after_layer:
            g = gain(blk.attn_in, model.cfg.d_model, dev)
            for name in ("q1", "k1", "q2", "k2", "v"):
                if hasattr(a, name):
                    yield (j, f"attn.{name}"), eff(getattr(a, name)) * g
        if j > after_layer or (j == after_layer and after_comp == "attn"):
            g = gain(blk.mlp_in, model.cfg.d_model, dev)
            yield (j, "mlp.l"), eff(blk.mlp.l) * g
            yield (j, "mlp.r"), eff(blk.mlp.r) * g
    g = gain(model.final_norm, model.cfg.d_model, dev)
    yield (len(model.blocks), "unembed"), upcast(model.unembed.weight.detach())[: model.cfg.vocab_size] * g


@torch.no_grad()
def read_write_graph(model, top_k: int = 5, threshold: float = 0.2, layer_window: int | None = None):
    edges, summary = [], []
    for (i, comp), W, oscope in _writers(model):
        Wn = W / W.norm(dim=0, keepdim=True).clamp_min(1e-30)
        for (j, rname), Rm in _readers(model, i, comp, layer_window):
            raw = Rm @ W
            cos = (Rm / Rm.norm(dim=1, keepdim=True).clamp_min(1e-30)) @ Wn
            a = cos.abs()
            row = {"writer": f"L{i}.{comp}", "reader": f"L{j}.{rname}", "writer_output_norm": oscope,
                   "max_abs_cos": float(a.max()), "mean_abs_cos": float(a.mean()),
                   "frac_abs_cos_gt": float((a > threshold).float().mean()), "threshold": threshold,
                   "raw_fro": float(raw.norm())}
            summary.append(row)
            if rname != "unembed":
                vals, flat = a.flatten().topk(min(top_k, a.numel()))
                for v, f in zip(vals, flat):
                    r_, c_ = divmod(int(f), a.shape[1])
                    edges.append({"writer": row["writer"], "write_col": c_, "reader": row["reader"], "read_row": r_,
                                  "cos": float(cos[r_, c_]), "raw": float(raw[r_, c_])})
    agg = {"pairs": len(summary), "edges_exported": len(edges), "layer_window": layer_window,
           "max_abs_cos": max(s["max_abs_cos"] for s in summary),
           "note": "content view only; overlap != usage. Direct residual path is identity (not listed)."}
    return agg, (summary, edges)


# ---------------------------------------------------------------------------------- 3. normalizer sensitivity
@torch.no_grad()
def _capture(model, idx, doc):
    inputs, hidden, mids, hooks = {}, [], [], []
    for name, m in dynamic_norms(model):
        hooks.append(m.register_forward_pre_hook(lambda mod, args, name=name: inputs.__setitem__(name, args[0].detach())))
    for blk in model.blocks:
        hooks.append(blk.register_forward_pre_hook(lambda mod, args: hidden.append([args[0].detach()])))
    for blk in model.blocks:
        target = blk.mlp_in if not isinstance(blk.mlp_in, nn.Identity) else blk.mlp
        hooks.append(target.register_forward_pre_hook(lambda mod, args: mids.append(args[0].detach())))
    _set_mode(model, "record")
    try:
        logits = model(idx, doc)
    finally:
        for h in hooks:
            h.remove()
    for h, mid in zip(hidden, mids):
        h.append(mid)
    return logits, inputs, {name: m.denom_saved for name, m in dynamic_norms(model)}, hidden


def _analytic_jvp(norm, x, delta):
    g = upcast(norm.weight.detach())
    if isinstance(norm, GroupRMSNorm):
        xs, ds = x.unflatten(-1, (norm.groups, -1)), delta.unflatten(-1, (norm.groups, -1))
    else:
        xs, ds = x[..., None, :], delta[..., None, :]
    dg = xs.shape[-1]
    r = torch.sqrt(xs.square().mean(-1, keepdim=True) + norm.eps)
    direct = (ds / r).flatten(-2) * g
    radial = (-(xs * (xs * ds).sum(-1, keepdim=True)) / (dg * r ** 3)).flatten(-2) * g
    return direct, radial


def normalizer_sensitivity(model, inputs, denoms, doc, max_tokens: int = 512) -> dict:
    gen = torch.Generator(device="cpu").manual_seed(1)
    valid = doc >= 0
    dpos = doc_positions(doc)
    sites = {}
    for name, m in dynamic_norms(model):
        if name not in inputs:
            continue
        x, r = upcast(inputs[name]), upcast(denoms[name])
        rv = r[..., 0] if r.shape[-1] == 1 else r.unflatten(-1, (m.groups, -1))[..., 0]
        by_pos = {}
        for lo, hi in POS_BUCKETS:
            sel = valid & (dpos >= lo) & (dpos < hi)
            if sel.any():
                by_pos[f"pos{lo}-{hi if hi < 1 << 29 else 'inf'}"] = float(rv[sel].float().median())
        xs = x[valid][:max_tokens]
        delta = torch.randn(xs.shape, generator=gen).to(xs.device, xs.dtype)
        direct, radial = _analytic_jvp(m, xs, delta)
        prev = m.denom_mode
        m.denom_mode = None
        _, auto = torch.func.jvp(lambda t: upcast(m(t)), (xs,), (delta,))
        m.denom_mode = prev
        ana, auto = (direct + radial).detach(), auto.detach()
        ratio = radial.detach().norm(dim=-1) / direct.detach().norm(dim=-1).clamp_min(1e-30)
        sites[name] = {"scope": norm_scope(m), "denominator": _quantiles(rv[valid]), "median_by_doc_position": by_pos,
                       "jvp_rel_err_analytic_vs_autograd": float((ana - auto).norm() / auto.norm().clamp_min(1e-30)),
                       "radial_over_direct_random_delta": _quantiles(ratio)}
    return {"sites": sites,
            "note": "radial term = denominator-mediated sensitivity; zero direct content edge does not imply no influence"}


# ---------------------------------------------------------------------------------- 4. ablation
@torch.no_grad()
def ablation_decomposition(model, batches) -> dict:
    comps = [(i, c) for i in range(len(model.blocks)) for c in ("attn", "mlp")]
    acc = {ic: {"live": [], "clamped": [], "keys": []} for ic in comps}
    for idx, doc, tgt in batches:
        _set_mode(model, "record")
        _, base = _token_losses(model, idx, doc, tgt)
        keys, valid = _doc_keys(doc, tgt)
        for i, c in comps:
            model.blocks[i].ablate = frozenset({c})
            _set_mode(model, None)
            _, live = _token_losses(model, idx, doc, tgt)
            _set_mode(model, "clamp")
            _, clamped = _token_losses(model, idx, doc, tgt)
            model.blocks[i].ablate = frozenset()
            acc[(i, c)]["live"].append((live - base)[valid])
            acc[(i, c)]["clamped"].append((clamped - base)[valid])
            acc[(i, c)]["keys"].append(keys)
        _set_mode(model, None)
    res = {}
    for (i, c), a in acc.items():
        nm = [l - k for l, k in zip(a["live"], a["clamped"])]
        res[f"L{i}.{c}"] = {"dCE_live": _paired_doc_stats(a["live"], a["keys"]),
                            "dCE_norm_clamped": _paired_doc_stats(a["clamped"], a["keys"]),
                            "norm_mediated(live-clamped)": _paired_doc_stats(nm, a["keys"])}
    return {"components": res, "uncertainty": "standard error across documents, not across seeds",
            "note": "softmax row normalization is not clamped" if model.cfg.attention == "softmax"
            else "all dynamic norms clamped"}


# ---------------------------------------------------------------------------------- 5. fixed denominators
def _row_hashes(batches) -> set:
    out = set()
    for idx, doc, _ in batches:
        for r in range(idx.shape[0]):
            out.add(hashlib.sha256(idx[r].cpu().numpy().tobytes() + doc[r].cpu().numpy().tobytes()).hexdigest())
    return out


@torch.no_grad()
def fixed_denominator(model, batches) -> dict:
    op_class = model.operator_audit()["class"]
    sites = dynamic_norms(model)
    if not sites:
        return {"skipped": "no dynamic RMS/GroupRMS denominators to fix; this intervention is the identity",
                "operator_class": op_class,
                "note": "class comes from the operator audit; other dynamic operations (e.g. softmax) are untouched"}
    half = len(batches) // 2
    calib, evalb = (batches, batches) if len(batches) < 2 else (batches[:half], batches[half:])
    overlap = len(_row_hashes(calib) & _row_hashes(evalb))
    if len(batches) < 2:
        provenance = "in-sample: single probe batch used for both calibration and evaluation"
    elif overlap:
        provenance = f"overlapping: {overlap} identical (tokens, doc layout) rows in calibration and evaluation halves"
    else:
        provenance = "row-disjoint halves (no identical rows); not a document-level held-out guarantee"
    sums = {n: 0 for n, _ in sites}
    cnt = 0
    for idx, doc, _ in calib:
        _set_mode(model, "record")
        model(idx, doc)
        v = doc >= 0
        for n, m in sites:
            sums[n] = sums[n] + upcast(m.denom_saved)[v].sum(0)
        cnt += int(v.sum())
    _set_mode(model, None)
    n_targets = sum(int((t != -100).sum()) for _, _, t in evalb)
    base = {"operator_class": op_class, "calibration_tokens": cnt, "evaluation_targets": n_targets,
            "fit_eval_provenance": provenance, "targeted_sites": len(sites)}
    if cnt == 0 or n_targets == 0:
        return {**base, "skipped": "no calibration tokens" if cnt == 0 else "no scored evaluation targets"}
    for n, m in sites:
        m.denom_const = sums[n] / cnt
    stats = {"ce_live": [], "ce_fixed": [], "kl": [], "abs_logit_err": [], "top1_agree": []}
    for idx, doc, tgt in evalb:
        _set_mode(model, None)
        ll, cel = _token_losses(model, idx, doc, tgt)
        _set_mode(model, "const")
        lf, cef = _token_losses(model, idx, doc, tgt)
        v = tgt != -100
        lp, lq = F.log_softmax(ll, -1), F.log_softmax(lf, -1)
        kl = (lp.exp() * (lp - lq)).sum(-1)
        stats["ce_live"].append(cel[v])
        stats["ce_fixed"].append(cef[v])
        stats["kl"].append(kl[v])
        stats["abs_logit_err"].append((ll - lf).abs().mean(-1)[v])
        stats["top1_agree"].append((ll.argmax(-1) == lf.argmax(-1)).float()[v])
    _set_mode(model, None)
    metrics = {k: float(torch.cat(v).mean()) for k, v in stats.items()}
    out = {**base, **{k: (x if math.isfinite(x) else None) for k, x in metrics.items()}}
    bad = sorted(k for k, x in metrics.items() if not math.isfinite(x))
    if bad:
        out["nonfinite_metrics"] = bad
    out["note"] = "small average error on this distribution does not establish OOD/long-context equivalence"
    return out


# ---------------------------------------------------------------------------------- 6. low rank
def stable_rank(s: torch.Tensor) -> float:
    s = s.abs()
    return float(s.square().sum() / s.max().square().clamp_min(1e-30))


def entropy_rank(s: torch.Tensor) -> float:
    p = s.abs() / s.abs().sum().clamp_min(1e-30)
    p = p[p > 0]
    return float(torch.exp(-(p * p.log()).sum()))


@torch.no_grad()
def low_rank_structure(model, batches, n_dirs: int = 4, max_dense: int = 4096) -> dict:
    cfg = model.cfg
    d = cfg.d_model
    tg = torch.cat([b[2][b[2] >= 0].flatten() for b in batches])
    top = torch.bincount(tg, minlength=cfg.vocab_size).topk(3).indices.tolist()
    U_out = upcast(model.unembed.weight.detach()) * gain(model.final_norm, d, tg.device)
    logit_dirs = {f"logit[{top[0]}]-logit[{top[1]}]": U_out[top[0]] - U_out[top[1]],
                  f"logit[{top[0]}]-logit[{top[2]}]": U_out[top[0]] - U_out[top[2]]}
    mlps = []
    for i, blk in enumerate(model.blocks):
        if blk.mlp.kind == "swiglu":
            continue
        g = gain(blk.mlp_in, d, tg.device)
        L, R, D = eff(blk.mlp.l) * g, eff(blk.mlp.r) * g, eff(blk.mlp.d)
        Us = torch.linalg.svd(D, full_matrices=False).U[:, :n_dirs].T
        dirs = {**{f"D_sv{k}": Us[k] for k in range(Us.shape[0])}, **logit_dirs}
        row = {}
        for nm, u in dirs.items():
            if d > max_dense:
                row[nm] = {"skipped": f"d_model {d} > {max_dense}; use randomized eigensolver"}
                continue
            w = D.T @ u
            Q = L.T @ (w[:, None] * R)
            ev = torch.linalg.eigvalsh(0.5 * (Q + Q.T))
            o = ev.abs().argsort(descending=True)
            row[nm] = {"stable_rank": stable_rank(ev), "entropy_rank": entropy_rank(ev),
                       "top_eigs": [float(x) for x in ev[o[:8]]],
                       "frac_negative_mass": float(ev[ev < 0].abs().sum() / ev.abs().sum())}
        mlps.append({"layer": i, "forms": row})
    heads = []
    for i, blk in enumerate(model.blocks):
        a = blk.attn
        g = gain(blk.attn_in, d, tg.device)
        for pair in (("q1", "k1"), ("q2", "k2")):
            if not hasattr(a, pair[0]):
                continue
            Wq, Wk = eff(getattr(a, pair[0])) * g, eff(getattr(a, pair[1])) * g
            for h in range(cfg.heads):
                sl = slice(h * cfg.d_key, (h + 1) * cfg.d_key)
                s = torch.linalg.svdvals(torch.linalg.qr(Wq[sl].T).R @ torch.linalg.qr(Wk[sl].T).R.T)
                heads.append({"layer": i, "pair": "".join(pair), "head": h, "stable_rank": stable_rank(s),
                              "top_sv": float(s.max())})
    return {"mlp_quadratic_forms": mlps, "qk_forms": heads,
            "note": "compare across seeds before interpreting; quadratic forms are gauge-invariant, raw factors are not"}


# ---------------------------------------------------------------------------------- shared: probe scores
@torch.no_grad()
def probe_attention_scores(model, idx, doc, max_tokens: int = 512):
    """Scores S = q.k / sqrt(dk) (after RoPE) of every polynomial layer on the first probe row,
    the MLP sublayer inputs, and the (T, T) visibility mask."""
    cfg = model.cfg
    idx, doc = idx[:1, :max_tokens], doc[:1, :max_tokens]
    attn_in, mlp_in, hooks = {}, {}, []
    for i, blk in enumerate(model.blocks):
        hooks.append(blk.attn.register_forward_pre_hook(lambda m, a, i=i: attn_in.__setitem__(i, a[0].detach())))
        hooks.append(blk.mlp.register_forward_pre_hook(lambda m, a, i=i: mlp_in.__setitem__(i, a[0].detach())))
    try:
        with reference_path(model):
            model(idx, doc)
    finally:
        for h in hooks:
            h.remove()
    cos, sin = rope_tables(doc_positions(doc), cfg.d_key, cfg.rope_base)
    scores = []
    for i, blk in enumerate(model.blocks):
        a, x = blk.attn, upcast(attn_in[i])
        row = {}
        if a.kind != "softmax":
            heads = lambda lin: upcast(apply_rope(a._split_heads(x, lin, cfg.d_key), cos, sin))[0]  # noqa: E731
            row["S1"] = heads(a.q1) @ heads(a.k1).transpose(-1, -2) / cfg.d_key ** 0.5
            if hasattr(a, "q2"):
                row["S2"] = heads(a.q2) @ heads(a.k2).transpose(-1, -2) / cfg.d_key ** 0.5
        scores.append(row)
    return scores, mlp_in, visible_mask(doc)[0, 0]


# ---------------------------------------------------------------------------------- 7. stability
@torch.no_grad()
def stability_stats(model, idx, doc, max_tokens: int = 512) -> dict:
    scores, mlp_in, vis = probe_attention_scores(model, idx, doc, max_tokens)
    idx = idx[:1, :max_tokens]
    out = []
    for i, blk in enumerate(model.blocks):
        row = {"layer": i}
        if scores[i]:
            S1 = scores[i]["S1"]
            S2 = scores[i].get("S2", S1)
            for name, t in (("S1", S1), ("S2", S2), ("S1S2", S1 * S2)):
                v = t[:, vis]
                row[f"{name}_max_abs"] = float(v.abs().max())
                row[f"{name}_rms"] = float(v.square().mean().sqrt())
        m = blk.mlp
        if m.kind != "swiglu":
            z = upcast(mlp_in[i])
            prod = upcast(m.l(z)) * upcast(m.r(z))
            c = prod - prod.mean()
            row["mlp_prod_rms"] = float(prod.square().mean().sqrt())
            row["mlp_prod_max_abs"] = float(prod.abs().max())
            row["mlp_prod_excess_kurtosis"] = float(c.pow(4).mean() / c.square().mean().clamp_min(1e-30) ** 2 - 3)
        out.append(row)
    worst = {k: max(r.get(k, 0.0) for r in out) for k in ("S1S2_max_abs", "mlp_prod_max_abs", "mlp_prod_excess_kurtosis")}
    return {"per_layer": out, "worst": worst, "tokens": int(idx.shape[1]),
            "note": "single-row probe; track across checkpoints/scales rather than reading absolute values"}


def analyze(model, batches, out_dir: str, rw_layer_window: int | None = None) -> dict:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    was_training = model.training
    model.eval()
    batches = list(batches)
    if not batches:
        raise ValueError("analyze needs at least one probe batch")
    with reference_path(model), _restore_modes(model):
        idx, doc, _ = batches[0]
        _, inputs, denoms, hidden = _capture(model, idx, doc)
        audit = model.operator_audit()
        result = {"operator_class": audit["class"],
                  "normalizer_scopes": {n: norm_scope(m) for n, m in model.named_modules()
                                        if isinstance(m, (RMSNorm, GroupRMSNorm, LaggedRMS, TaperRMS))},
                  "local_tensor": local_tensor_check(model, hidden)}
        agg, (summary, edges) = read_write_graph(model, layer_window=rw_layer_window)
        result["read_write_graph"] = agg
        (out / "read_write_summary.json").write_text(json.dumps(summary))
        (out / "read_write_top_edges.json").write_text(json.dumps(edges))
        result["normalizer_sensitivity"] = normalizer_sensitivity(model, inputs, denoms, doc)
        result["ablation"] = ablation_decomposition(model, batches)
        result["fixed_denominator"] = fixed_denominator(model, batches)
        result["low_rank"] = low_rank_structure(model, batches)
        result["stability"] = stability_stats(model, idx, doc)
        result["files"] = ["read_write_summary.json", "read_write_top_edges.json", "analysis.json"]
    model.train(was_training)
    result = json.loads(json.dumps(result, default=float).replace("NaN", "null"))
    (out / "analysis.json").write_text(json.dumps(result, indent=1))
    return result


def analyze_checkpoint(cfg, checkpoint, out, *, batches=2, context=None, max_seconds=300.0, device="cpu",
                       run_budget_usd=None, rw_layer_window=None) -> dict:
    """Billed, frozen-state-checked ``analyze`` of a checkpoint on validation probe batches (the
    reference's ``analyze`` command, tnlm/cli.py:117-270): the model, its buffers, module modes,
    hooks and the probe batches must be unchanged afterwards; the probe plan, overlap audit and
    source provenance are written beside the diagnostics."""
    import hashlib
    import json
    import time

    from .budget import SpendLedger
    from .checkpoint import load_checkpoint
    from .config import Config
    from .data import (PackedSampler, audit_validation_overlap, batch_hash, manifest_hash,
                       validate_tokenizer_compatibility)
    from .evaluate import _training_descriptor
    from .models.model import TensorLM
    from .runtime import evaluation_validator
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    project, data = cfg.raw.get("project", {}), cfg.raw.get("data", {})
    context = data.get("context", 512) if context is None else context
    if rw_layer_window is not None and (type(rw_layer_window) is not int or rw_layer_window < 0):
        raise ValueError("rw_layer_window must be a nonnegative integer")
    if batches <= 0 or context <= 0 or max_seconds <= 0:
        raise ValueError("analysis requires positive batches, context and runtime cap")
    if project.get("dry_run", True):
        return {"dry_run": True, "command": "analyze", "checkpoint": str(checkpoint), "context": context,
                "batches": batches, "max_seconds": max_seconds, "rw_layer_window": rw_layer_window}
    out = Path(out)
    if out.exists():
        raise FileExistsError(f"analysis output already exists: {out}")
    dev = torch.device(device)
    rate = project.get("gpu_hourly_rate_usd")
    if rate is None or (dev.type == "cuda" and rate <= 0):
        raise ValueError("declare actual gpu_hourly_rate_usd (explicit 0 allowed for CPU)")
    ledger = SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                         project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets"))
    run_id = str(out.resolve())
    ledger.begin(run_id, rate, max_seconds, run_budget_usd, parent_checkpoint=str(checkpoint),
                 cost_margin_fraction=project.get("cost_margin_fraction", .1), stage=project.get("stage", "A"))
    started, status = time.monotonic(), "failed"
    try:
        evaluation = cfg.raw.get("evaluation", {})
        manifest = evaluation.get("validation_manifest", data.get("manifest"))
        tok_compat = validate_tokenizer_compatibility(data["manifest"], manifest, allow_test_only=dev.type == "cpu")
        sampler = PackedSampler(manifest, split="val", context=context, batch_size=data.get("micro_batch_size", 1),
                                seed=int(evaluation.get("seed", 0)))
        model = TensorLM(cfg.model).to(dev)
        payload = load_checkpoint(checkpoint, model, expected_manifest_hash=manifest_hash(data["manifest"]),
                                  config_validator=evaluation_validator(cfg), restore_rng=False, map_location="cpu")
        code, ckpt_progress = payload["code"], payload["progress"]
        descriptor = _training_descriptor(payload)
        del payload
        model.eval()

        def fingerprint():
            h = hashlib.sha256()
            for name, t in list(model.named_parameters()) + list(model.named_buffers()):
                h.update(name.encode())
                h.update(str((t.dtype, tuple(t.shape))).encode())
                h.update(t.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes())
            return h.hexdigest()

        def lifecycle():
            return ({n: (m.training, getattr(m, "collecting", None), getattr(m, "denom_mode", None),
                         getattr(m, "ablate", None), tuple(m._forward_hooks), tuple(m._forward_pre_hooks))
                     for n, m in model.named_modules()},
                    {n: p.requires_grad for n, p in model.named_parameters()})
        before_state, before_modes = fingerprint(), lifecycle()
        initial = sampler.state_dict()
        probe, mappings = [], []
        for _ in range(batches):
            if time.monotonic() - started >= max_seconds:
                raise TimeoutError("analysis runtime cap during probe setup")
            probe.append(tuple(t.to(dev) for t in sampler.next_batch()))
            mappings.append(sampler.batch_mappings())
        hashes = [batch_hash(b) for b in probe]
        plan = {"version": 1, "validation_manifest_sha256": manifest_hash(manifest), "split": "val",
                "context": context, "sampler_initial": initial, "batch_mappings": mappings, "batch_hashes": hashes}
        plan_sha = hashlib.sha256(json.dumps(plan, sort_keys=True, separators=(",", ":")).encode()).hexdigest()
        docs = {item["document_id"] for mapping in mappings for row in mapping for item in row["ranges"]
                if item["packed_token_start"] < row["input_length"]}
        audit = audit_validation_overlap(data["manifest"], manifest, document_ids=docs)
        if audit["has_overlap"]:
            raise ValueError("analysis validation has exact whole-document content overlap")
        seed = int(evaluation.get("seed", 0))
        devices = [dev.index if dev.index is not None else torch.cuda.current_device()] if dev.type == "cuda" else []
        with torch.random.fork_rng(devices=devices):
            torch.random.default_generator.manual_seed(seed)
            if devices:
                torch.cuda.default_generators[devices[0]].manual_seed(seed)
            result = analyze(model, probe, str(out), **({} if rw_layer_window is None else
                                                          {"rw_layer_window": rw_layer_window}))
        if [batch_hash(b) for b in probe] != hashes:
            raise RuntimeError("analysis changed probe batch inputs or targets")
        after_state, after_modes = fingerprint(), lifecycle()
        if before_state != after_state or before_modes != after_modes:
            raise RuntimeError("analysis changed model state, modes, collection flags, gradient flags or hooks")
        pkg = Path(__file__).parent
        sources = {str(p.relative_to(pkg)): hashlib.sha256(p.read_bytes()).hexdigest() for p in sorted(pkg.rglob("*.py"))}
        provenance = {"checkpoint": str(Path(checkpoint).resolve()), "training_descriptor": descriptor,
                      "checkpoint_progress": ckpt_progress, "checkpoint_code": code,
                      "checkpoint_manifest_sha256": hashlib.sha256((Path(checkpoint) / "manifest.json").read_bytes()).hexdigest(),
                      "validation_manifest_sha256": manifest_hash(manifest), "split": "val", "batches": batches,
                      "context": context, "rw_layer_window": rw_layer_window, "probe_seed": seed,
                      "runtime_source_sha256": sources, "batch_hashes": hashes, "probe_plan": plan,
                      "probe_plan_sha256": plan_sha, "data_overlap_audit": audit, "tokenizer_compatibility": tok_compat,
                      "frozen_state": {"before": before_state, "after": after_state, "unchanged": True},
                      "sampler": sampler.state_dict(), "runtime_cap_seconds": max_seconds}
        result["training_descriptor"] = descriptor
        result["evaluation_provenance"] = provenance
        json.dumps(result, allow_nan=False)
        out.mkdir(parents=True, exist_ok=True)
        (out / "invocation.json").write_text(json.dumps(provenance, indent=2))
        status = "complete"
    finally:
        ledger.finish(run_id, time.monotonic() - started, status)
    result["billing"] = json.loads(ledger.path.read_text())["runs"][run_id]
    (out / "analysis-invocation-result.json").write_text(json.dumps(result, indent=2, allow_nan=False))
    return result
