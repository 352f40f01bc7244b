"""Scaling-law grid: plan, run and fit (the reference's scripts/scaling_grid.py and
scripts/fit_scaling_law.py workflow).

    python -m tensor_train_ing_b200.runbook.scaling plan GRID.yaml [--tpp 5 10 20 40]
    python -m tensor_train_ing_b200.runbook.scaling run GRID.yaml SIZE --out runs/grid [--device cuda]
    python -m tensor_train_ing_b200.runbook.scaling fit runs/grid [--params total|non_embedding] [--compute 1e20 ...]

``GRID.yaml`` holds ``base`` (a full run config) and ``sizes`` (name -> ``{model: {...}, lr: x}``).
For a size with N total parameters and tokens-per-parameter budgets r, each budget is
D_r = r N rounded to the update batch.  One constant-LR parent trains to the 90 % point of the
largest budget and saves a milestone at the 90 % point of every budget; each budget then gets a
cooldown branch from its milestone (linear decay over the last 10 %, ending exactly at D_r) and a
held-out evaluation.  Sharing the parent costs max(D) plus about 10 % of each budget instead of
the sum of the budgets.  Every stage is skipped when its ``result.json`` / ``evaluation.json``
exists, so an interrupted grid resumes where it stopped.

The fit is Hoffmann et al. (2022), approach 3: L(N, D) = E + A / N^alpha + B / D^beta, fitted by
minimising the Huber loss (delta 1e-3) between log L and
log(exp(a - alpha log N) + exp(b - beta log D) + exp(e)) with L-BFGS from a grid of starting
points (A = e^a, B = e^b, E = e^e).  Under C = 6 N D the loss-optimal split is
N_opt = G (C / 6)^(beta / (alpha + beta)), D_opt = C / (6 N_opt), G = (alpha A / (beta B))^(1 / (alpha + beta)).
"""
from __future__ import annotations

import argparse
import copy
import itertools
import json
import math
import sys
from pathlib import Path

import torch
import yaml

from ..config import Config, ModelConfig
from ..models.shapes import count_params


# ====================================================================================== plan
def _params(model: dict) -> dict:
    fields = ModelConfig.__dataclass_fields__
    return count_params(ModelConfig(**{k: v for k, v in model.items() if k in fields}))


def plan_size(grid: dict, size: str, tpps=(5, 10, 20, 40), out_root="runs/scaling_grid") -> dict:
    """The size's config, budgets, milestones and branch points."""
    if size not in grid["sizes"]:
        raise ValueError(f"unknown size {size!r}; the grid has {sorted(grid['sizes'])}")
    spec = grid["sizes"][size]
    cfg = copy.deepcopy(grid["base"])
    cfg.setdefault("model", {}).update(spec.get("model", {}))
    cfg.setdefault("train", {}).update(spec.get("train", {}))
    if "lr" in spec:
        cfg["train"]["lr"] = spec["lr"]
    counts = _params(cfg["model"])
    batch = int(cfg["train"]["global_prediction_tokens_per_update"])
    budgets = sorted({max(1, round(r * counts["total"] / batch)) * batch for r in tpps})
    branch = {d: -(-(9 * d // 10) // batch) * batch for d in budgets}
    if any(branch[d] >= d or branch[d] <= 0 for d in budgets):
        raise ValueError(f"a budget is too small for a 10% cooldown at batch {batch}: {budgets}")
    cfg["train"]["rung_total_tokens"] = budgets[-1]
    cfg["train"]["schedule"] = "constant_with_separate_cooldown"
    cfg.setdefault("project", {})["milestone_tokens"] = sorted({9 * d // 10 for d in budgets})
    out = Path(out_root) / size
    cfg["project"].setdefault("spend_ledger", str(out / "spend.json"))
    parent_tokens = branch[budgets[-1]]
    return {"size": size, "out": str(out), "config": cfg, "params": counts, "batch": batch, "budgets": budgets,
            "branch_tokens": {str(d): branch[d] for d in budgets},
            "tokens_per_param": {str(d): d / counts["total"] for d in budgets},
            "parent_tokens": parent_tokens,
            "trained_tokens": parent_tokens + sum(d - branch[d] for d in budgets)}


# ====================================================================================== run
def _done(run_dir: Path, name="result.json") -> dict | None:
    try:
        return json.loads((run_dir / name).read_text())
    except (OSError, ValueError):
        return None


def run_size(plan: dict, *, device="cuda", max_seconds=86_400.0, bootstrap_samples=200) -> dict:
    """Parent, then per budget a cooldown branch from its milestone and an evaluation."""
    from ..evaluate import evaluate_checkpoint
    from ..train import train_run
    out = Path(plan["out"])
    out.mkdir(parents=True, exist_ok=True)
    cfg_path = out / "config.yaml"
    if cfg_path.exists() and yaml.safe_load(cfg_path.read_text()) != plan["config"]:
        raise ValueError(f"{cfg_path} holds another configuration; move it aside to start over")
    cfg_path.write_text(yaml.safe_dump(plan["config"], sort_keys=False))
    cfg = Config.from_yaml(str(cfg_path))
    batch = plan["batch"]
    parent = out / "parent"
    if _done(parent) is None:
        steps = plan["parent_tokens"] // batch
        train_run(cfg, parent, max_steps=steps, max_seconds=max_seconds, device=device)
    report = {"size": plan["size"], "budgets": []}
    for d in plan["budgets"]:
        branch = plan["branch_tokens"][str(d)]
        milestone = parent / f"milestone-{9 * d // 10:012d}"
        stage = out / f"{plan['size']}_tpp{d / plan['params']['total']:g}"
        cooled, evaluation = stage / "cooldown", stage / "evaluation"
        if _done(cooled) is None:
            horizon = -(-(d - branch) // batch)
            train_run(cfg, cooled, max_steps=horizon, max_seconds=max_seconds, device=device, resume=str(milestone),
                      cooldown_steps=horizon, cooldown_end_tokens=d)
        ev = _done(evaluation, "evaluation.json")
        if ev is None:
            ev = evaluate_checkpoint(cfg, _done(cooled)["checkpoint"], evaluation, max_seconds=max_seconds,
                                     device=device, bootstrap_samples=bootstrap_samples)
        report["budgets"].append({"tokens": d, "ce": ev["ce"], "evaluation": str(evaluation / "evaluation.json")})
    return report


# ====================================================================================== fit
def collect(root, params="total") -> list[tuple[float, float, float, str]]:
    """(N, D, CE, name) of every evaluated branch below ``root`` (one directory per size holding its
    ``config.yaml``); D is the branch's own trained-token endpoint."""
    points = []
    for size_dir in sorted(Path(root).iterdir()):
        if not (size_dir / "config.yaml").exists():
            continue
        n = float(_params(yaml.safe_load((size_dir / "config.yaml").read_text())["model"])[params])
        for ev in sorted(size_dir.glob("*/evaluation/evaluation.json")):
            report = json.loads(ev.read_text())
            points.append((n, float(report["training_descriptor"]["actual_prediction_tokens"]), float(report["ce"]),
                           ev.parent.parent.name))
    return points


def _log_model(theta, log_n, log_d):
    a, b, e, alpha, beta = theta
    return torch.logsumexp(torch.stack([a - alpha * log_n, b - beta * log_d, e.expand_as(log_n)]), dim=0)


FIT_STARTS = tuple(itertools.product((0.0, 5.0, 10.0, 15.0), (0.0, 5.0, 10.0, 15.0), (-1.0, 0.0, 1.0, 1.5),
                                     (0.0, 0.5, 1.0), (0.0, 0.5, 1.0)))  # (a, b, e, alpha, beta)


def fit(points, delta: float = 1e-3, starts=FIT_STARTS) -> dict:
    """Fit L = E + A / N^alpha + B / D^beta to ``points`` = [(N, D, L), ...]."""
    n, d, loss = (torch.tensor([p[i] for p in points], dtype=torch.float64) for i in range(3))
    log_n, log_d, log_l = n.log(), d.log(), loss.log()
    best = (math.inf, None)
    for start in starts:
        theta = torch.tensor(start, dtype=torch.float64, requires_grad=True)
        opt = torch.optim.LBFGS([theta], lr=1.0, max_iter=200, line_search_fn="strong_wolfe")

        def objective():
            opt.zero_grad()
            value = torch.nn.functional.huber_loss(_log_model(theta, log_n, log_d), log_l, delta=delta,
                                                   reduction="sum")
            value.backward()
            return value
        try:
            opt.step(objective)
        except RuntimeError:
            continue
        with torch.no_grad():
            value = float(torch.nn.functional.huber_loss(_log_model(theta, log_n, log_d), log_l, delta=delta,
                                                         reduction="sum"))
        if math.isfinite(value) and value < best[0]:
            best = (value, theta.detach().clone())
    if best[1] is None:
        raise ValueError("no starting point converged")
    a, b, e, alpha, beta = best[1].tolist()
    return {"A": math.exp(a), "B": math.exp(b), "E": math.exp(e), "alpha": alpha, "beta": beta, "huber": best[0]}


def compute_optimal(law: dict, compute: float) -> dict:
    """Loss-optimal parameters and tokens for a budget of ``compute`` = 6 N D FLOPs."""
    alpha, beta = law["alpha"], law["beta"]
    g = (alpha * law["A"] / (beta * law["B"])) ** (1.0 / (alpha + beta))
    n = g * (compute / 6.0) ** (beta / (alpha + beta))
    d = compute / 6.0 / n
    return {"compute": compute, "N_opt": n, "D_opt": d, "tokens_per_param": d / n,
            "L_opt": law["E"] + law["A"] / n ** alpha + law["B"] / d ** beta}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = p.add_subparsers(dest="cmd", required=True)
    pl = sub.add_parser("plan")
    pl.add_argument("grid")
    pl.add_argument("--tpp", type=float, nargs="+", default=[5, 10, 20, 40])
    pl.add_argument("--tokens-per-second", type=float, help="measured rate, for GPU-hour estimates")
    rn = sub.add_parser("run")
    rn.add_argument("grid")
    rn.add_argument("size")
    rn.add_argument("--out", default="runs/scaling_grid")
    rn.add_argument("--tpp", type=float, nargs="+", default=[5, 10, 20, 40])
    rn.add_argument("--device", default="cuda")
    rn.add_argument("--max-seconds", type=float, default=86_400.0)
    ft = sub.add_parser("fit")
    ft.add_argument("root")
    ft.add_argument("--params", choices=["total", "non_embedding"], default="total")
    ft.add_argument("--compute", type=float, nargs="*", default=[1e19, 1e20, 1e21, 1e22])
    a = p.parse_args(argv)
    if a.cmd == "plan":
        grid = yaml.safe_load(Path(a.grid).read_text())
        for size in grid["sizes"]:
            plan = plan_size(grid, size, a.tpp)
            hours = plan["trained_tokens"] / a.tokens_per_second / 3600 if a.tokens_per_second else None
            print(json.dumps({k: plan[k] for k in ("size", "params", "budgets", "parent_tokens", "trained_tokens")}
                             | {"gpu_hours": hours}))
        return 0
    if a.cmd == "run":
        grid = yaml.safe_load(Path(a.grid).read_text())
        print(json.dumps(run_size(plan_size(grid, a.size, a.tpp, a.out), device=a.device, max_seconds=a.max_seconds),
                         indent=1))
        return 0
    points = collect(a.root, a.params)
    sizes = sorted({pt[0] for pt in points})
    for n, d, ce, name in points:
        print(f"  {name:24s} N={n / 1e6:8.1f}M D={d / 1e9:7.3f}B tokens/param={d / n:6.1f} CE={ce:.4f}")
    if len(sizes) < 3 or len(points) < 6:
        print("a five-parameter fit needs at least 3 sizes and 6 points")
        return 1
    law = fit([pt[:3] for pt in points])
    print(json.dumps({"law": law, "optimal": [compute_optimal(law, c) for c in a.compute]}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
