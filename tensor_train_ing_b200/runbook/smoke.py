"""Trainer smoke on a prepared dataset: train, resume, check the replay, evaluate (the reference's
scripts/h100_trainer_smoke.py role).

    python -m tensor_train_ing_b200.runbook.smoke --config run.yaml --out runs/smoke [--steps 4] [--device cuda]

Runs the serial trainer for ``2 * steps`` updates in one go and, separately, ``steps`` updates
followed by a resume for ``steps`` more; the two final checkpoints must hold identical weights
(bitwise: the kernels reduce in a fixed order).  Then the final checkpoint is evaluated on the
held-out split.  The report (``smoke.json`` in ``--out``) gives both trajectories' losses, the replay
verdict, the evaluation CE and the throughput of the uninterrupted run.  The config must not be a
dry run; its spend ledger records the four runs.
"""
from __future__ import annotations

import argparse
import copy
import json
import sys
from pathlib import Path

import torch


def _losses(run_dir: Path) -> list[float]:
    return [json.loads(x)["loss"] for x in (run_dir / "metrics.jsonl").read_text().splitlines()]


def run_smoke(cfg, out_dir, *, steps=4, device="cuda", max_seconds=3600.0, bootstrap_samples=100) -> dict:
    from ..checkpoint import verified_state_path
    from ..config import Config
    from ..evaluate import evaluate_checkpoint
    from ..train import train_run
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    if cfg.raw.get("project", {}).get("dry_run", True):
        raise ValueError("the smoke trains: set project.dry_run to false")
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=False)
    full = train_run(copy.deepcopy(cfg), out / "full", max_steps=2 * steps, max_seconds=max_seconds, device=device)
    first = train_run(copy.deepcopy(cfg), out / "first", max_steps=steps, max_seconds=max_seconds, device=device)
    resumed = train_run(copy.deepcopy(cfg), out / "resumed", max_steps=steps, max_seconds=max_seconds, device=device,
                        resume=first["checkpoint"])
    a = torch.load(verified_state_path(full["checkpoint"]), map_location="cpu", weights_only=False)["model"]
    b = torch.load(verified_state_path(resumed["checkpoint"]), map_location="cpu", weights_only=False)["model"]
    differing = sorted(k for k in a if not torch.equal(a[k], b[k]))
    evaluation = evaluate_checkpoint(copy.deepcopy(cfg), full["checkpoint"], out / "evaluation",
                                     max_seconds=max_seconds, device=device, bootstrap_samples=bootstrap_samples)
    rows = [json.loads(x) for x in (out / "full" / "metrics.jsonl").read_text().splitlines()]
    later = rows[1:] or rows
    report = {"status": "passed" if not differing else "failed", "device": device, "steps": 2 * steps,
              "uninterrupted_losses": _losses(out / "full"),
              "interrupted_losses": _losses(out / "first") + _losses(out / "resumed"),
              "replay_bitwise_identical": not differing, "differing_tensors": differing[:20],
              "evaluation_ce": evaluation["ce"], "evaluation_prediction_tokens": evaluation["prediction_tokens"],
              "tokens_per_second_after_first_update": sum(r["prediction_tokens"] for r in later)
              / sum(r["seconds"] for r in later),
              "fused_sm100a_path": full.get("operator_audit") is not None and device.startswith("cuda")}
    (out / "smoke.json").write_text(json.dumps(report, indent=2) + "\n")
    return report


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--config", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--device", default="cuda")
    p.add_argument("--max-seconds", type=float, default=3600.0)
    a = p.parse_args(argv)
    report = run_smoke(a.config, a.out, steps=a.steps, device=a.device, max_seconds=a.max_seconds)
    print(json.dumps({k: report[k] for k in ("status", "replay_bitwise_identical", "evaluation_ce")}))
    return 0 if report["status"] == "passed" else 1


if __name__ == "__main__":
    sys.exit(main())
