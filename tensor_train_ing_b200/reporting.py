"""Bounded summaries and loss-curve plots of completed training-run segments (reference
tnlm/reporting.py:9-118).

``summarize_runs`` writes ``comparison.json`` / ``comparison.csv`` (one row of cost, identity and
training-evidence metadata per run) and three SVG plots (training CE against scored tokens, run
elapsed time and billed USD).  The plots are written directly as SVG polylines, so no plotting
library is needed.  Training cross entropy is not held-out quality; rows are never ranked.
"""
from __future__ import annotations

import csv
import json
import math
from pathlib import Path
from xml.sax.saxutils import escape

_COLORS = ("#1f77b4", "#ff7f0e", "#2ca02c", "#d62728", "#9467bd", "#8c564b", "#e377c2", "#7f7f7f")


def _svg_plot(curves, field, xlabel, path, width=600, height=400):
    """Line plot of loss against ``field`` for each curve, with axes, ticks and a legend."""
    pts = [(p[field], p["loss"]) for c in curves for p in c["points"]
           if p.get(field) is not None and p.get("loss") is not None]
    left, right, top, bottom = 70, 20, 20, 50
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" '
           f'viewBox="0 0 {width} {height}" font-family="sans-serif" font-size="11">',
           f'<rect width="{width}" height="{height}" fill="white"/>']
    if pts:
        x0, x1 = min(p[0] for p in pts), max(p[0] for p in pts)
        y0, y1 = min(p[1] for p in pts), max(p[1] for p in pts)
        x1 = x1 if x1 > x0 else x0 + 1
        y1 = y1 if y1 > y0 else y0 + 1
        sx = lambda v: left + (v - x0) / (x1 - x0) * (width - left - right)  # noqa: E731
        sy = lambda v: height - bottom - (v - y0) / (y1 - y0) * (height - top - bottom)  # noqa: E731
        out.append(f'<line x1="{left}" y1="{height - bottom}" x2="{width - right}" y2="{height - bottom}" stroke="black"/>')
        out.append(f'<line x1="{left}" y1="{top}" x2="{left}" y2="{height - bottom}" stroke="black"/>')
        for i in range(5):
            xv, yv = x0 + (x1 - x0) * i / 4, y0 + (y1 - y0) * i / 4
            out.append(f'<text x="{sx(xv):.1f}" y="{height - bottom + 15}" text-anchor="middle">{xv:.4g}</text>')
            out.append(f'<text x="{left - 5}" y="{sy(yv) + 4:.1f}" text-anchor="end">{yv:.4g}</text>')
            out.append(f'<line x1="{left}" y1="{sy(yv):.1f}" x2="{width - right}" y2="{sy(yv):.1f}" '
                       'stroke="#ddd" stroke-width="0.5"/>')
        for k, c in enumerate(curves):
            line = [(sx(p[field]), sy(p["loss"])) for p in c["points"]
                    if p.get(field) is not None and p.get("loss") is not None]
            if not line:
                continue
            color = _COLORS[k % len(_COLORS)]
            out.append(f'<polyline fill="none" stroke="{color}" stroke-width="1.5" points="'
                       + " ".join(f"{x:.1f},{y:.1f}" for x, y in line) + '"/>')
            out.append(f'<text x="{width - right - 5}" y="{top + 14 * (k + 1)}" text-anchor="end" fill="{color}">'
                       f'{escape(c["label"])}</text>')
    out.append(f'<text x="{(left + width - right) / 2}" y="{height - 10}" text-anchor="middle">{escape(xlabel)}</text>')
    out.append(f'<text x="15" y="{(top + height - bottom) / 2}" text-anchor="middle" '
               f'transform="rotate(-90 15 {(top + height - bottom) / 2})">Training cross entropy</text>')
    out.append("</svg>")
    Path(path).write_text("\n".join(out) + "\n")


def summarize_runs(run_dirs, out_dir, *, max_plot_points=2000):
    """Export cost / identity metadata and training-loss curves of completed run segments.

    Elapsed time and cost are per segment; token positions include inherited training; the
    parent checkpoint stays explicit."""
    if max_plot_points < 2:
        raise ValueError("max_plot_points must be at least two")
    table, curves = [], []
    for directory in run_dirs:
        directory = Path(directory).resolve()
        result = json.loads((directory / "result.json").read_text())
        ledger = json.loads(Path(result["spend_ledger"]).read_text())
        billing = ledger["runs"][result["run_id"]]
        if billing["status"] != "complete":
            raise ValueError(f"cannot summarize unfinished run: {directory}")
        metrics = directory / "metrics.jsonl"
        lines = metrics.read_text().splitlines() if metrics.exists() else []
        stride = max(1, math.ceil(len(lines) / max_plot_points))
        points, last, seg_tokens, step_seconds = [], None, 0, 0.0
        for i, line in enumerate(lines):
            rec = json.loads(line)
            last = rec
            seg_tokens += rec["prediction_tokens"]
            step_seconds += rec["seconds"]
            if i % stride == 0 or i == len(lines) - 1:
                points.append({k: rec.get(k) for k in ("step", "tokens", "loss", "run_elapsed_seconds",
                                                       "run_billed_usd")})
        progress = result["progress"]
        desc = result.get("training_descriptor", {})
        if not isinstance(desc, dict) or desc.get("source") != "checkpoint_payload" or desc.get("version") != 1:
            desc = {}
        train_cfg = result.get("train_config", {})
        table.append({
            "run": str(directory), "operator_class": result["operator_audit"]["class"],
            "normalization": result["model_config"]["normalization"], "optimizer": train_cfg.get("optimizer"),
            "configured_lr": train_cfg.get("lr"), "seed": desc.get("seed"), "width": desc.get("width"),
            "depth": desc.get("depth"), "schedule": desc.get("schedule", "unknown"),
            "cooldown_status": desc.get("cooldown_status", "unknown"),
            "completion_status": desc.get("completion_status", "unknown"),
            "segment_target_prediction_tokens": desc.get("segment_target_prediction_tokens"),
            "cooldown_steps": desc.get("cooldown_steps"), "aux_adamw_lr": train_cfg.get("aux_adamw_lr"),
            "attention": result["model_config"]["attention"], "parameters": result["parameters"]["total"],
            "context": result["data"]["context"], "context_history": desc.get("context_history"),
            "context_history_status": desc.get("context_history_status", "unknown"),
            "data_manifest_sha256": result["data"]["manifest_sha256"],
            "global_prediction_tokens": progress["tokens"], "run_prediction_tokens": seg_tokens,
            "trajectory_calibration_tokens": progress.get("calibration", {}).get("tokens", 0),
            "run_calibration_tokens": 0 if result.get("parent") else progress.get("calibration", {}).get("tokens", 0),
            "parent_checkpoint": result.get("parent"), "final_training_ce": last["loss"] if last else None,
            "run_billed_usd": billing["spent_usd"], "run_elapsed_seconds": billing["elapsed_seconds"],
            "step_average_prediction_tokens_per_second": seg_tokens / step_seconds if step_seconds else None,
            "cuda_peak_allocated_bytes": result.get("cuda_peak_allocated_bytes"),
            "cuda_peak_reserved_bytes": result.get("cuda_peak_reserved_bytes"),
            "device": result["runtime"]["device"], "compile_enabled": result.get("compile_enabled", False),
            "warmup_dominates_completed_segment": result.get("warmup_dominates_completed_segment")})
        curves.append({"run": str(directory), "label": directory.name, "points": points,
                       "original_metric_points": len(lines)})
    if not table:
        raise ValueError("at least one completed run is required")
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=False)
    bundle = {"runs": table, "curves": curves, "metric": "training cross entropy; not held-out model quality",
              "context_scope": "context is the current segment; context_history records known earlier segments",
              "schedule_scope": "cooldown and completion labels come from checkpoint training evidence; mixed "
                                "schedules or horizons are not automatically comparable",
              "automatic_ranking_eligible": False,
              "step_timing_scope": "all recorded steps; use profile for a declared warm-up exclusion",
              "cost_scope": "per run segment, including setup and checkpoints; parent cost is not combined",
              "interpretation_scope": "operator classification only; use analyze for measured diagnostics"}
    (out / "comparison.json").write_text(json.dumps(bundle, indent=2, allow_nan=False))
    with (out / "comparison.csv").open("w", newline="") as f:
        writer = csv.DictWriter(f, fieldnames=list(table[0]))
        writer.writeheader()
        writer.writerows(table)
    for field, label, name in (("tokens", "Global scored prediction tokens", "loss-vs-tokens.svg"),
                               ("run_elapsed_seconds", "Run elapsed seconds (includes setup)", "loss-vs-time.svg"),
                               ("run_billed_usd", "Run billed USD", "loss-vs-cost.svg")):
        _svg_plot(curves, field, label, out / name)
    return {"output": str(out), "runs": len(table), "artifacts": sorted(p.name for p in out.iterdir()),
            "metric": bundle["metric"], "cost_scope": bundle["cost_scope"]}
