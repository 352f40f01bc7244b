"""Interpretability diagnostics of a trained TensorLM, written as one JSON report.

Sections of ``analyze(model, batches, out_dir)`` (same measurements and report schema as the
reference's analysis, tnlm/analysis.py:29-596):

  local tensors        the bilinear MLP as a symmetric coefficient tensor restricted to a random
                       subspace (it reproduces the module exactly) and, for plain RMSNorm inputs,
                       with the norm's gain folded in on probe activations;
  read/write graph     cosine overlaps between upstream write directions (O, D columns) and
                       downstream read vectors (Q, K, V, L, R rows and the unembedding);
  normalizer sensitivity  per-site denominators, analytic vs autograd JVPs, radial/direct ratio;
  ablation             branch removal with live vs clamped denominators, per-document paired;
  fixed denominators   calibrated constant denominators against live ones on held-out rows;
  low rank             MLP quadratic forms along output/logit directions, per-head QK forms;
  stability            max |S|, |S1 S2| and bilinear-product tails (shared with QK-clip).

Every diagnostic runs the model's module path, where norms expose their denominators and hooks
see every sublayer; the model, its buffers, modes and hooks are left as they were.
"""
from __future__ import annotations

import hashlib
import json
import math
import time
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
QUANTILE_SAMPLE = 1_000_000


# ====================================================================================== model views
@contextmanager
def reference_path(model):
    """Run the model through its module path (hooks and denominator modes visible)."""
    forced = getattr(model, "_force_reference", False)
    model._force_reference = True
    try:
        yield model
    finally:
        model._force_reference = forced


def eff(lin: nn.Module) -> torch.Tensor:
    """The matrix a linear layer applies, detached, in the reduction dtype."""
    return upcast((lin.effective_weight() if isinstance(lin, SpectralLinear) else lin.weight).detach())


def gain(norm: nn.Module, d: int, device) -> torch.Tensor:
    """The fixed per-feature map a norm site contributes, which folds into the adjacent linear maps.
    A TaperRMS part-way through its taper has none and is refused."""
    if isinstance(norm, TaperRMS):
        g = float(norm.gate)
        if g == 1.0:
            return upcast(norm.weight.detach())
        if g == 0.0 and bool(norm.frozen):
            return float(norm.c) * upcast(norm.weight_tilde.detach())
        raise ValueError(f"a TaperRMS at gate {g} (frozen={bool(norm.frozen)}) has no fixed map to fold")
    w = getattr(norm, "weight", None)
    if w is None:  # nn.Identity
        return torch.ones(d, device=device)
    g = upcast(w.detach())
    if isinstance(norm, LaggedRMS):
        g = g / torch.sqrt(norm.mean_sq.detach().to(g.dtype) + norm.eps)
    return g


def norm_scope(norm: nn.Module) -> str:
    """What a norm site divides by, in words."""
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


class Denominators:
    """Switch every dynamic norm of a model between live, record, clamp and const denominators;
    leaving the context resets modes, saved and constant denominators, and branch ablations."""

    def __init__(self, model):
        self.model = model
        self.sites = dynamic_norms(model)

    def mode(self, mode):
        for _, m in self.sites:
            m.denom_mode = mode

    def saved(self) -> dict:
        return {name: m.denom_saved for name, m in self.sites}

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        for _, m in self.sites:
            m.denom_mode, m.denom_saved, m.denom_const = None, None, None
        for blk in self.model.blocks:
            blk.ablate = frozenset()
        return False


def _quantiles(x: torch.Tensor) -> dict:
    x = upcast(x.flatten())
    if x.numel() == 0:
        return {}
    if x.numel() > QUANTILE_SAMPLE:
        x = x[torch.randperm(x.numel(), device=x.device)[:QUANTILE_SAMPLE]]
    qs = torch.quantile(x, torch.tensor(QUANTILES, device=x.device, dtype=x.dtype))
    return {**{f"q{int(p * 100):02d}": float(v) for p, v in zip(QUANTILES, qs)}, "mean": float(x.mean())}


def _rel(a, b) -> float:
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _token_losses(model, idx, doc, tgt):
    logits = upcast(model(idx, doc))
    per_token = F.cross_entropy(logits.flatten(0, 1), tgt.flatten(), ignore_index=-100, reduction="none")
    return logits, per_token.view_as(tgt)


class PairedDocs:
    """Per-token differences grouped by document: the summary is the mean over documents of each
    document's mean difference, with its standard error across documents."""

    def __init__(self):
        self.parts: list[tuple[torch.Tensor, torch.Tensor]] = []

    @staticmethod
    def keys(doc, tgt):
        """(document key of every scored token, scored mask); keys are unique across rows."""
        scored = tgt != -100
        key = torch.arange(doc.shape[0], device=doc.device)[:, None] * (doc.max() + 2) + doc.clamp_min(0)
        return key[scored], scored

    def add(self, diffs, keys):
        self.parts.append((diffs, keys))

    def summary(self) -> dict:
        means = []
        for d, k in self.parts:
            uniq, inv = torch.unique(k, return_inverse=True)
            sums = torch.zeros(len(uniq), device=d.device, dtype=torch.float64).index_add_(0, inv, d.double())
            counts = torch.zeros(len(uniq), device=d.device, dtype=torch.float64).index_add_(
                0, inv, torch.ones_like(d, dtype=torch.float64))
            means.append(sums / counts)
        v = torch.cat(means)
        n = v.numel()
        return {"mean": float(v.mean()), "doc_se": float(v.std(unbiased=True) / math.sqrt(n)) if n > 1 else float("nan"),
                "documents": n}


# ====================================================================================== 1. local tensors
@torch.no_grad()
def mlp_local_tensor(blk, basis: torch.Tensor, fold_gain: bool = True):
    """The symmetrised coefficient tensor (d_out, k[+1], k[+1]) of a block's MLP on span(basis); an
    affine MLP gets one more coordinate carrying its biases."""
    m = blk.mlp
    L, R, D = eff(m.l), eff(m.r), eff(m.d)
    if fold_gain:
        g = gain(blk.mlp_in, L.shape[1], L.device)
        L, R = L * g, R * g
    basis = basis.to(L.dtype)
    LU, RU = L @ basis, R @ basis
    if m.l.bias is not None:
        one = torch.zeros(1, LU.shape[1] + 1, device=LU.device, dtype=LU.dtype)
        one[0, -1] = 1
        LU = torch.cat([torch.cat([LU, upcast(m.l.bias.detach())[:, None]], 1), one])
        RU = torch.cat([torch.cat([RU, upcast(m.r.bias.detach())[:, None]], 1), one])
        D = torch.cat([D, upcast(m.d.bias.detach())[:, None]], 1)
    T = torch.einsum("oh,ha,hb->oab", D, LU, RU)
    return 0.5 * (T + T.transpose(1, 2))


@torch.no_grad()
def local_tensor_check(model, hidden, k: int = 8, n: int = 16) -> dict:
    gen = torch.Generator(device="cpu").manual_seed(0)
    d = model.cfg.d_model
    rows = []
    for i, blk in enumerate(model.blocks):
        if blk.mlp.kind == "swiglu":
            rows.append({"layer": i, "skipped": "SwiGLU is class G"})
            continue
        dev, dt = blk.mlp.l.weight.device, upcast(blk.mlp.l.weight).dtype
        U = torch.linalg.qr(torch.randn(d, k, generator=gen, dtype=torch.float64)).Q.to(device=dev, dtype=dt)
        z = torch.randn(n, k, generator=gen, dtype=torch.float64).to(device=dev, dtype=dt)
        T = mlp_local_tensor(blk, U, fold_gain=False)
        coords = torch.cat([z, torch.ones(n, 1, device=dev, dtype=dt)], 1) if T.shape[1] > k else z
        rebuilt = torch.einsum("oab,na,nb->no", T, coords, coords)
        row = {"layer": i, "subspace_rank": k,
               "rel_err_restricted_tensor": _rel(rebuilt, upcast(blk.mlp(z @ U.T)))}
        norm = blk.mlp_in
        if type(norm) is RMSNorm and blk.mlp.kind == "bilinear":
            # with the gain folded into L and R the MLP of the normalised input is a quadratic form
            # of x divided by r(x)^2
            x = upcast(hidden[i][1].reshape(-1, d)[:256])
            g = gain(norm, d, dev)
            r = torch.sqrt(x.square().mean(-1, keepdim=True) + norm.eps)
            L, R, D = eff(blk.mlp.l), eff(blk.mlp.r), eff(blk.mlp.d)
            folded = (((x * g) @ L.T) * ((x * g) @ R.T)) @ D.T / r ** 2
            row["rel_err_gain_folded_on_probe"] = _rel(folded, upcast(blk.mlp(norm(x))))
        rows.append(row)
    return {"per_layer": rows, "max_rel_err": max((r.get("rel_err_restricted_tensor", 0) for r in rows), default=0.0)}


# ====================================================================================== 2. read/write graph
def _writers(model):
    """(layer, component), the write matrix with its output-norm gain, and the norm's scope."""
    for i, blk in enumerate(model.blocks):
        for comp, lin, out_norm in (("attn", blk.attn.o, blk.attn_out), ("mlp", blk.mlp.d, blk.mlp_out)):
            W = eff(lin)
            if isinstance(out_norm, DynamicNorm):
                W = W * gain(out_norm, W.shape[0], W.device)[:, None]
            yield (i, comp), W, norm_scope(out_norm)


def _readers(model, after_layer, after_comp, layer_window=None):
    """Read matrices (with their input-norm gains) of every sublayer downstream of a writer."""
    dev, d = model.unembed.weight.device, model.cfg.d_model
    for j, blk in enumerate(model.blocks):
        if layer_window is not None and j > after_layer + layer_window:
            break
        if j > after_layer:
            g = gain(blk.attn_in, d, dev)
            for lin_name in ("q1", "k1", "q2", "k2", "v"):
                if hasattr(blk.attn, lin_name):
                    yield (j, f"attn.{lin_name}"), eff(getattr(blk.attn, lin_name)) * g
        if j > after_layer or (j == after_layer and after_comp == "attn"):
            g = gain(blk.mlp_in, d, dev)
            yield (j, "mlp.l"), eff(blk.mlp.l) * g
            yield (j, "mlp.r"), eff(blk.mlp.r) * g
    g = gain(model.final_norm, d, dev)
    yield (len(model.blocks), "unembed"), upcast(model.unembed.weight.detach())[: model.cfg.vocab_size] * g


@torch.no_grad()
def read_write_graph(model, top_k: int = 5, threshold: float = 0.2, layer_window: int | None = None):
    pairs, edges = [], []
    for (i, comp), W, scope in _writers(model):
        W_unit = W / W.norm(dim=0, keepdim=True).clamp_min(1e-30)
        for (j, reader), Rm in _readers(model, i, comp, layer_window):
            raw = Rm @ W
            cos = (Rm / Rm.norm(dim=1, keepdim=True).clamp_min(1e-30)) @ W_unit
            mag = cos.abs()
            pair = {"writer": f"L{i}.{comp}", "reader": f"L{j}.{reader}", "writer_output_norm": scope,
                    "max_abs_cos": float(mag.max()), "mean_abs_cos": float(mag.mean()),
                    "frac_abs_cos_gt": float((mag > threshold).float().mean()), "threshold": threshold,
                    "raw_fro": float(raw.norm())}
            pairs.append(pair)
            if reader == "unembed":
                continue
            vals, flat = mag.flatten().topk(min(top_k, mag.numel()))
            for _v, f in zip(vals, flat):
                r_, c_ = divmod(int(f), mag.shape[1])
                edges.append({"writer": pair["writer"], "write_col": c_, "reader": pair["reader"], "read_row": r_,
                              "cos": float(cos[r_, c_]), "raw": float(raw[r_, c_])})
    overview = {"pairs": len(pairs), "edges_exported": len(edges), "layer_window": layer_window,
                "max_abs_cos": max(p["max_abs_cos"] for p in pairs),
                "note": "content view only; overlap != usage. Direct residual path is identity (not listed)."}
    return overview, (pairs, edges)


# ====================================================================================== 3. normalizer sensitivity
@torch.no_grad()
def _capture(model, idx, doc, dens: Denominators):
    """One recorded forward: every dynamic norm's input and denominator, and per block its input
    and the MLP sublayer's input."""
    norm_inputs, hidden, mids, hooks = {}, [], [], []
    for name, m in dens.sites:
        hooks.append(m.register_forward_pre_hook(lambda mod, args, name=name: norm_inputs.__setitem__(name, args[0].detach())))
    for blk in model.blocks:
        hooks.append(blk.register_forward_pre_hook(lambda mod, args: hidden.append([args[0].detach()])))
    for blk in model.blocks:
        target = blk.mlp_in if not isinstance(blk.mlp_in, nn.Identity) else blk.mlp
        hooks.append(target.register_forward_pre_hook(lambda mod, args: mids.append(args[0].detach())))
    dens.mode("record")
    try:
        logits = model(idx, doc)
    finally:
        for h in hooks:
            h.remove()
    for h, mid in zip(hidden, mids):
        h.append(mid)
    return logits, norm_inputs, dens.saved(), hidden


def _analytic_jvp(norm, x, delta):
    """(direct, radial) parts of the (group) RMSNorm JVP: delta/r and the divisor's response."""
    g = upcast(norm.weight.detach())
    groups = norm.groups if isinstance(norm, GroupRMSNorm) else 1
    xs, ds = x.unflatten(-1, (groups, -1)), delta.unflatten(-1, (groups, -1))
    dg = xs.shape[-1]
    r = torch.sqrt(xs.square().mean(-1, keepdim=True) + norm.eps)
    direct = (ds / r).flatten(-2) * g
    radial = (-(xs * (xs * ds).sum(-1, keepdim=True)) / (dg * r ** 3)).flatten(-2) * g
    return direct, radial


def normalizer_sensitivity(model, inputs, denoms, doc, max_tokens: int = 512) -> dict:
    gen = torch.Generator(device="cpu").manual_seed(1)
    valid, dpos = doc >= 0, doc_positions(doc)
    sites = {}
    for name, m in dynamic_norms(model):
        if name not in inputs:
            continue
        x, r = upcast(inputs[name]), upcast(denoms[name])
        per_token = r[..., 0] if r.shape[-1] == 1 else r.unflatten(-1, (m.groups, -1))[..., 0]
        by_pos = {}
        for lo, hi in POS_BUCKETS:
            sel = valid & (dpos >= lo) & (dpos < hi)
            if sel.any():
                by_pos[f"pos{lo}-{hi if hi < 1 << 29 else 'inf'}"] = float(per_token[sel].float().median())
        xs = x[valid][:max_tokens]
        delta = torch.randn(xs.shape, generator=gen).to(xs.device, xs.dtype)
        direct, radial = _analytic_jvp(m, xs, delta)
        mode, m.denom_mode = m.denom_mode, None
        _, autograd = torch.func.jvp(lambda t: upcast(m(t)), (xs,), (delta,))
        m.denom_mode = mode
        ratio = radial.detach().norm(dim=-1) / direct.detach().norm(dim=-1).clamp_min(1e-30)
        sites[name] = {"scope": norm_scope(m), "denominator": _quantiles(per_token[valid]),
                       "median_by_doc_position": by_pos,
                       "jvp_rel_err_analytic_vs_autograd": _rel((direct + radial).detach(), autograd.detach()),
                       "radial_over_direct_random_delta": _quantiles(ratio)}
    return {"sites": sites,
            "note": "radial term = denominator-mediated sensitivity; zero direct content edge does not imply no influence"}


# ====================================================================================== 4. ablation
@torch.no_grad()
def ablation_decomposition(model, batches) -> dict:
    dens = Denominators(model)
    comps = [(i, c) for i in range(len(model.blocks)) for c in ("attn", "mlp")]
    live = {ic: PairedDocs() for ic in comps}
    clamped = {ic: PairedDocs() for ic in comps}
    mediated = {ic: PairedDocs() for ic in comps}
    for idx, doc, tgt in batches:
        dens.mode("record")
        _, base = _token_losses(model, idx, doc, tgt)
        keys, scored = PairedDocs.keys(doc, tgt)
        for i, c in comps:
            model.blocks[i].ablate = frozenset({c})
            dens.mode(None)
            _, with_live = _token_losses(model, idx, doc, tgt)
            dens.mode("clamp")
            _, with_clamp = _token_losses(model, idx, doc, tgt)
            model.blocks[i].ablate = frozenset()
            d_live, d_clamp = (with_live - base)[scored], (with_clamp - base)[scored]
            live[(i, c)].add(d_live, keys)
            clamped[(i, c)].add(d_clamp, keys)
            mediated[(i, c)].add(d_live - d_clamp, keys)
        dens.mode(None)
    comps_out = {f"L{i}.{c}": {"dCE_live": live[(i, c)].summary(), "dCE_norm_clamped": clamped[(i, c)].summary(),
                               "norm_mediated(live-clamped)": mediated[(i, c)].summary()} for i, c in comps}
    return {"components": comps_out, "uncertainty": "standard error across documents, not across seeds",
            "note": "softmax row normalization is not clamped" if model.cfg.attention == "softmax"
            else "all dynamic norms clamped"}


# ====================================================================================== 5. fixed denominators
def _row_hashes(batches) -> set:
    return {hashlib.sha256(idx[r].cpu().numpy().tobytes() + doc[r].cpu().numpy().tobytes()).hexdigest()
            for idx, doc, _ in batches for r in range(idx.shape[0])}


def _split_provenance(batches):
    if len(batches) < 2:
        return batches, batches, "in-sample: single probe batch used for both calibration and evaluation"
    half = len(batches) // 2
    fit, held = batches[:half], batches[half:]
    shared = len(_row_hashes(fit) & _row_hashes(held))
    if shared:
        return fit, held, f"overlapping: {shared} identical (tokens, doc layout) rows in calibration and evaluation halves"
    return fit, held, "row-disjoint halves (no identical rows); not a document-level held-out guarantee"


@torch.no_grad()
def fixed_denominator(model, batches) -> dict:
    op_class = model.operator_audit()["class"]
    dens = Denominators(model)
    if not dens.sites:
        return {"skipped": "no dynamic RMS/GroupRMS denominators to fix; this intervention is the identity",
                "operator_class": op_class,
                "note": "class comes from the operator audit; other dynamic operations (e.g. softmax) are untouched"}
    fit, held, provenance = _split_provenance(batches)
    sums = {name: 0 for name, _ in dens.sites}
    tokens = 0
    for idx, doc, _ in fit:
        dens.mode("record")
        model(idx, doc)
        real = doc >= 0
        for name, m in dens.sites:
            sums[name] = sums[name] + upcast(m.denom_saved)[real].sum(0)
        tokens += int(real.sum())
    dens.mode(None)
    targets = sum(int((t != -100).sum()) for _, _, t in held)
    base = {"operator_class": op_class, "calibration_tokens": tokens, "evaluation_targets": targets,
            "fit_eval_provenance": provenance, "targeted_sites": len(dens.sites)}
    if tokens == 0 or targets == 0:
        return {**base, "skipped": "no calibration tokens" if tokens == 0 else "no scored evaluation targets"}
    for name, m in dens.sites:
        m.denom_const = sums[name] / tokens
    parts = {"ce_live": [], "ce_fixed": [], "kl": [], "abs_logit_err": [], "top1_agree": []}
    for idx, doc, tgt in held:
        dens.mode(None)
        live_logits, live_ce = _token_losses(model, idx, doc, tgt)
        dens.mode("const")
        fixed_logits, fixed_ce = _token_losses(model, idx, doc, tgt)
        scored = tgt != -100
        lp, lq = F.log_softmax(live_logits, -1), F.log_softmax(fixed_logits, -1)
        parts["ce_live"].append(live_ce[scored])
        parts["ce_fixed"].append(fixed_ce[scored])
        parts["kl"].append((lp.exp() * (lp - lq)).sum(-1)[scored])
        parts["abs_logit_err"].append((live_logits - fixed_logits).abs().mean(-1)[scored])
        parts["top1_agree"].append((live_logits.argmax(-1) == fixed_logits.argmax(-1)).float()[scored])
    dens.mode(None)
    metrics = {k: float(torch.cat(v).mean()) for k, v in parts.items()}
    out = {**base, **{k: (x if math.isfinite(x) else None) for k, x in metrics.items()}}
    bad = sorted(k for k, x in metrics.items() if not math.isfinite(x))
    if bad:
        out["nonfinite_metrics"] = bad
    out["note"] = "small average error on this distribution does not establish OOD/long-context equivalence"
    return out


# ====================================================================================== 6. low rank
def stable_rank(s: torch.Tensor) -> float:
    """sum s^2 / max s^2."""
    s = s.abs()
    return float(s.square().sum() / s.max().square().clamp_min(1e-30))


def entropy_rank(s: torch.Tensor) -> float:
    """exp of the entropy of |s| normalised to a distribution."""
    p = s.abs() / s.abs().sum().clamp_min(1e-30)
    p = p[p > 0]
    return float(torch.exp(-(p * p.log()).sum()))


def _form_spectrum(ev) -> dict:
    order = ev.abs().argsort(descending=True)
    return {"stable_rank": stable_rank(ev), "entropy_rank": entropy_rank(ev),
            "top_eigs": [float(x) for x in ev[order[:8]]],
            "frac_negative_mass": float(ev[ev < 0].abs().sum() / ev.abs().sum())}


@torch.no_grad()
def low_rank_structure(model, batches, n_dirs: int = 4, max_dense: int = 4096) -> dict:
    cfg = model.cfg
    d = cfg.d_model
    targets = torch.cat([b[2][b[2] >= 0].flatten() for b in batches])
    top = torch.bincount(targets, minlength=cfg.vocab_size).topk(3).indices.tolist()
    U_out = upcast(model.unembed.weight.detach()) * gain(model.final_norm, d, targets.device)
    logit_dirs = {f"logit[{top[0]}]-logit[{top[1]}]": U_out[top[0]] - U_out[top[1]],
                  f"logit[{top[0]}]-logit[{top[2]}]": U_out[top[0]] - U_out[top[2]]}
    mlps = []
    for i, blk in enumerate(model.blocks):
        if blk.mlp.kind == "swiglu":
            continue
        g = gain(blk.mlp_in, d, targets.device)
        L, R, D = eff(blk.mlp.l) * g, eff(blk.mlp.r) * g, eff(blk.mlp.d)
        out_dirs = torch.linalg.svd(D, full_matrices=False).U[:, :n_dirs].T
        forms = {}
        for name, u in {**{f"D_sv{k}": out_dirs[k] for k in range(out_dirs.shape[0])}, **logit_dirs}.items():
            if d > max_dense:
                forms[name] = {"skipped": f"d_model {d} > {max_dense}; use randomized eigensolver"}
                continue
            Q = L.T @ ((D.T @ u)[:, None] * R)  # u . MLP(x) = x^T Q x
            forms[name] = _form_spectrum(torch.linalg.eigvalsh(0.5 * (Q + Q.T)))
        mlps.append({"layer": i, "forms": forms})
    heads = []
    for i, blk in enumerate(model.blocks):
        g = gain(blk.attn_in, d, targets.device)
        for n, (q_lin, k_lin) in enumerate(blk.attn.qk_pairs(), start=1):
            Wq, Wk = eff(q_lin) * g, eff(k_lin) * g
            for h in range(cfg.heads):
                rows = slice(h * cfg.d_key, (h + 1) * cfg.d_key)
                s = torch.linalg.svdvals(torch.linalg.qr(Wq[rows].T).R @ torch.linalg.qr(Wk[rows].T).R.T)
                heads.append({"layer": i, "pair": f"q{n}k{n}", "head": h, "stable_rank": stable_rank(s),
                              "top_sv": float(s.max())})
    return {"mlp_quadratic_forms": mlps, "qk_forms": heads,
            "note": "compare across seeds before interpreting; quadratic forms are gauge-invariant, raw factors are not"}


# ====================================================================================== shared: probe scores
@torch.no_grad()
def probe_attention_scores(model, idx, doc, max_tokens: int = 512):
    """Scores S = q.k / sqrt(dk) (after RoPE) of every polynomial layer on the first probe row, the
    MLP sublayer inputs, and the (T, T) visibility mask."""
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
    scale = cfg.d_key ** 0.5
    scores = []
    for i, blk in enumerate(model.blocks):
        a, x = blk.attn, upcast(attn_in[i])
        row = {}
        if a.kind != "softmax":
            heads = lambda lin: upcast(apply_rope(a._split_heads(x, lin, cfg.d_key), cos, sin))[0]  # noqa: E731
            for n, (q_lin, k_lin) in enumerate(a.qk_pairs(), start=1):
                row[f"S{n}"] = heads(q_lin) @ heads(k_lin).transpose(-1, -2) / scale
        scores.append(row)
    return scores, mlp_in, visible_mask(doc)[0, 0]


# ====================================================================================== 7. stability
@torch.no_grad()
def stability_stats(model, idx, doc, max_tokens: int = 512) -> dict:
    scores, mlp_in, vis = probe_attention_scores(model, idx, doc, max_tokens)
    out = []
    for i, blk in enumerate(model.blocks):
        row = {"layer": i}
        if scores[i]:
            S1 = scores[i]["S1"]
            S2 = scores[i].get("S2", S1)
            for name, t in (("S1", S1), ("S2", S2), ("S1S2", S1 * S2)):
                seen = t[:, vis]
                row[f"{name}_max_abs"] = float(seen.abs().max())
                row[f"{name}_rms"] = float(seen.square().mean().sqrt())
        if blk.mlp.kind != "swiglu":
            z = upcast(mlp_in[i])
            prod = upcast(blk.mlp.l(z)) * upcast(blk.mlp.r(z))
            centred = prod - prod.mean()
            row["mlp_prod_rms"] = float(prod.square().mean().sqrt())
            row["mlp_prod_max_abs"] = float(prod.abs().max())
            row["mlp_prod_excess_kurtosis"] = float(
                centred.pow(4).mean() / centred.square().mean().clamp_min(1e-30) ** 2 - 3)
        out.append(row)
    worst = {k: max(r.get(k, 0.0) for r in out) for k in ("S1S2_max_abs", "mlp_prod_max_abs", "mlp_prod_excess_kurtosis")}
    return {"per_layer": out, "worst": worst, "tokens": int(idx[:1, :max_tokens].shape[1]),
            "note": "single-row probe; track across checkpoints/scales rather than reading absolute values"}


# ====================================================================================== report
def analyze(model, batches, out_dir: str, rw_layer_window: int | None = None) -> dict:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    batches = list(batches)
    if not batches:
        raise ValueError("analyze needs at least one probe batch")
    was_training = model.training
    model.eval()
    with reference_path(model), Denominators(model) as dens:
        idx, doc, _ = batches[0]
        _, inputs, denoms, hidden = _capture(model, idx, doc, dens)
        result = {"operator_class": model.operator_audit()["class"],
                  "normalizer_scopes": {n: norm_scope(m) for n, m in model.named_modules()
                                        if isinstance(m, (RMSNorm, GroupRMSNorm, LaggedRMS, TaperRMS))},
                  "local_tensor": local_tensor_check(model, hidden)}
        overview, (pairs, edges) = read_write_graph(model, layer_window=rw_layer_window)
        result["read_write_graph"] = overview
        (out / "read_write_summary.json").write_text(json.dumps(pairs))
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


# ====================================================================================== checkpoint analysis
def _model_fingerprint(model) -> str:
    h = hashlib.sha256()
    for name, t in list(model.named_parameters()) + list(model.named_buffers()):
        h.update(name.encode())
        h.update(str((t.dtype, tuple(t.shape))).encode())
        h.update(t.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def _model_lifecycle(model):
    """Modes, collection flags, denominator modes, ablations, hooks and gradient flags."""
    return ({n: (m.training, getattr(m, "collecting", None), getattr(m, "denom_mode", None),
                 getattr(m, "ablate", None), tuple(m._forward_hooks), tuple(m._forward_pre_hooks))
             for n, m in model.named_modules()},
            {n: p.requires_grad for n, p in model.named_parameters()})


class _ProbePlan:
    """The validation batches an analysis runs on, their identity (plan + sha256) and the
    whole-document overlap audit against the training data."""

    def __init__(self, cfg, manifest, context, batches, device, deadline):
        from .data import PackedSampler, audit_validation_overlap, batch_hash, manifest_hash
        evaluation, data = cfg.raw.get("evaluation", {}), cfg.raw.get("data", {})
        self.seed = int(evaluation.get("seed", 0))
        self.sampler = PackedSampler(manifest, split="val", context=context,
                                     batch_size=data.get("micro_batch_size", 1), seed=self.seed)
        initial = self.sampler.state_dict()
        self.batches, mappings = [], []
        for _ in range(batches):
            if time.monotonic() >= deadline:
                raise TimeoutError("analysis runtime cap during probe setup")
            self.batches.append(tuple(t.to(device) for t in self.sampler.next_batch()))
            mappings.append(self.sampler.batch_mappings())
        self.hashes = [batch_hash(b) for b in self.batches]
        self.plan = {"version": 1, "validation_manifest_sha256": manifest_hash(manifest), "split": "val",
                     "context": context, "sampler_initial": initial, "batch_mappings": mappings,
                     "batch_hashes": self.hashes}
        self.sha256 = hashlib.sha256(json.dumps(self.plan, sort_keys=True, separators=(",", ":")).encode()).hexdigest()
        docs = {item["document_id"] for mapping in mappings for row in mapping for item in row["ranges"]
                if item["packed_token_start"] < row["input_length"]}
        self.audit = audit_validation_overlap(data["manifest"], manifest, document_ids=docs)
        if self.audit["has_overlap"]:
            raise ValueError("analysis validation has exact whole-document content overlap")

    def unchanged(self) -> bool:
        from .data import batch_hash
        return [batch_hash(b) for b in self.batches] == self.hashes


def analyze_checkpoint(cfg, checkpoint, out, *, batches=2, context=None, max_seconds=300.0, device="cpu",
                       run_budget_usd=None, rw_layer_window=None) -> dict:
    """``analyze`` of a checkpoint on validation probe batches, billed to the spend ledger, with the
    model's state, modes and hooks and the probe batches verified unchanged afterwards; the probe
    plan, overlap audit and source provenance are written beside the diagnostics (the reference's
    ``analyze`` command, tnlm/cli.py:117-270)."""
    from .budget import SpendLedger
    from .checkpoint import load_checkpoint
    from .config import Config
    from .data import manifest_hash, validate_tokenizer_compatibility
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
        manifest = cfg.raw.get("evaluation", {}).get("validation_manifest", data.get("manifest"))
        tok_compat = validate_tokenizer_compatibility(data["manifest"], manifest, allow_test_only=dev.type == "cpu")
        model = TensorLM(cfg.model).to(dev)
        payload = load_checkpoint(checkpoint, model, expected_manifest_hash=manifest_hash(data["manifest"]),
                                  config_validator=evaluation_validator(cfg), restore_rng=False, map_location="cpu")
        code, ckpt_progress, descriptor = payload["code"], payload["progress"], _training_descriptor(payload)
        del payload
        model.eval()
        state_before, modes_before = _model_fingerprint(model), _model_lifecycle(model)
        probe = _ProbePlan(cfg, manifest, context, batches, dev, started + max_seconds)
        cuda = [dev.index if dev.index is not None else torch.cuda.current_device()] if dev.type == "cuda" else []
        with torch.random.fork_rng(devices=cuda):
            torch.random.default_generator.manual_seed(probe.seed)
            if cuda:
                torch.cuda.default_generators[cuda[0]].manual_seed(probe.seed)
            kw = {} if rw_layer_window is None else {"rw_layer_window": rw_layer_window}
            result = analyze(model, probe.batches, str(out), **kw)
        if not probe.unchanged():
            raise RuntimeError("analysis changed probe batch inputs or targets")
        state_after = _model_fingerprint(model)
        if state_before != state_after or modes_before != _model_lifecycle(model):
            raise RuntimeError("analysis changed model state, modes, collection flags, gradient flags or hooks")
        pkg = Path(__file__).parent
        sources = {str(p.relative_to(pkg)): hashlib.sha256(p.read_bytes()).hexdigest() for p in sorted(pkg.rglob("*.py"))}
        provenance = {"checkpoint": str(Path(checkpoint).resolve()), "training_descriptor": descriptor,
                      "checkpoint_progress": ckpt_progress, "checkpoint_code": code,
                      "checkpoint_manifest_sha256": hashlib.sha256((Path(checkpoint) / "manifest.json").read_bytes()).hexdigest(),
                      "validation_manifest_sha256": manifest_hash(manifest), "split": "val", "batches": batches,
                      "context": context, "rw_layer_window": rw_layer_window, "probe_seed": probe.seed,
                      "runtime_source_sha256": sources, "batch_hashes": probe.hashes, "probe_plan": probe.plan,
                      "probe_plan_sha256": probe.sha256, "data_overlap_audit": probe.audit,
                      "tokenizer_compatibility": tok_compat,
                      "frozen_state": {"before": state_before, "after": state_after, "unchanged": True},
                      "sampler": probe.sampler.state_dict(), "runtime_cap_seconds": max_seconds}
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
