"""Paired-seed validation summaries from evaluation reports, no model execution (reference
tnlm/replication.py:61-225).

Each ``{seed, left, right}`` pair compares two conditions trained with the same seed on identical
validation targets.  Every declared difference between the conditions must be listed in
``allowed_between_dimensions`` (training-descriptor dimensions or full ``config.*`` paths); within a
condition only the seed may differ.  The aggregate is the equal-weight mean of per-seed deltas
with its sample SD / SE; no seed confidence interval, p-value or winner is reported.
"""
from __future__ import annotations

import hashlib
import json
import math
import statistics
from pathlib import Path

from .comparison_batch import _publish_json
from .evaluate import _training_comparison, compare_evaluations

_CONFIG_DIMENSIONS = {
    "optimizer": "train.optimizer", "width": "model.d_model", "depth": "model.layers", "train_context": "data.context",
    "rung_total_tokens": "train.rung_total_tokens",
    "global_prediction_tokens_per_update": "train.global_prediction_tokens_per_update", "lr": "train.lr",
    "normalization": "model.normalization", "attention": "model.attention", "aux_adamw_lr": "train.aux_adamw_lr",
    "schedule": "train.schedule",
    **{k: "model." + k for k in ("width_scaling_base", "width_lr_exponent", "width_logit_exponent",
                                 "depth_scaling_base", "depth_lr_exponent", "depth_residual_base",
                                 "depth_residual_exponent", "residual_alpha")},
    **{k: "train." + k for k in ("weight_decay_hidden", "beta1", "beta2")},
}


def _hash(value, name):
    if not isinstance(value, str) or len(value) != 64 or any(c not in "0123456789abcdef" for c in value):
        raise ValueError(f"{name} must be a SHA256 hex digest")
    return value


def _configuration(report, seed):
    value = report.get("training_descriptor", {}).get("configuration")
    if (not isinstance(value, dict) or not isinstance(value.get("model"), dict)
            or not isinstance(value.get("train"), dict) or "project" in value
            or type(value["train"].get("seed")) is not int or value["train"]["seed"] != seed):
        raise ValueError("complete checkpoint configuration with matching seed is required")
    return value


def _leaves(value, prefix="config"):
    if isinstance(value, dict):
        out = {}
        for k, v in value.items():
            if not isinstance(k, str) or "." in k:
                raise ValueError("configuration keys must be unambiguous dot-path components")
            out.update(_leaves(v, f"{prefix}.{k}"))
        return out if value else {prefix: {}}
    return {prefix: value}


def _differences(left, right, *, ignore_seed=False):
    a, b = _leaves(left), _leaves(right)
    if set(a) != set(b):
        raise ValueError("unknown/missing full configuration evidence paths")
    return [k for k in sorted(a) if not (ignore_seed and k == "config.train.seed")
            and (type(a[k]) is not type(b[k]) or a[k] != b[k])]


def compare_seed_pairs(pairs, out_dir, *, allowed_between_dimensions) -> dict:
    if not isinstance(pairs, list) or len(pairs) < 2:
        raise ValueError("at least two explicit seed pairs are required")
    allowed = allowed_between_dimensions
    if not isinstance(allowed, list) or any(not isinstance(v, str) for v in allowed) or len(set(allowed)) != len(allowed):
        raise ValueError("allowed_between_dimensions must be a unique list of dimension names")
    if "seed" in allowed or "config.train.seed" in allowed:
        raise ValueError("seed cannot be an allowed between-condition difference")
    cache, seeds, references, baseline, per_seed = {}, set(), {}, None, []
    ids = {s: {"model": set(), "state": set(), "manifest": set()} for s in ("left", "right")}
    dup_models = {"left": [], "right": []}

    def read(value):
        if not isinstance(value, (str, Path)):
            raise ValueError("seed-pair inputs must be evaluation report paths")
        path = Path(value).resolve()
        if path not in cache:
            raw = path.read_bytes()
            report = json.loads(raw)
            if not isinstance(report, dict):
                raise ValueError("evaluation report must be a JSON object")
            cache[path] = report, hashlib.sha256(raw).hexdigest()
        return cache[path][0], str(path), cache[path][1]
    for pair in pairs:
        if not isinstance(pair, dict) or set(pair) != {"seed", "left", "right"}:
            raise ValueError("each pair requires exactly seed, left and right")
        seed = pair["seed"]
        if type(seed) is not int or seed < 0 or seed in seeds:
            raise ValueError("pair seeds must be unique nonnegative integers")
        seeds.add(seed)
        loaded = {s: read(pair[s]) for s in ("left", "right")}
        reports = {s: v[0] for s, v in loaded.items()}
        comparison = compare_evaluations(reports["left"], reports["right"], None, bootstrap_samples=0)
        dims = comparison["training_comparison"]["dimensions"]
        configs = {s: _configuration(reports[s], seed) for s in ("left", "right")}
        paths = set(_leaves(configs["left"])) & set(_leaves(configs["right"]))
        if any(v not in dims and v not in paths for v in allowed):
            raise ValueError("unknown allowed training dimension or configuration path")
        full = _differences(configs["left"], configs["right"])
        mapped = {"config." + _CONFIG_DIMENSIONS[n] for n in allowed if n in _CONFIG_DIMENSIONS}
        undeclared = set(full) - set(allowed) - mapped
        if undeclared:
            raise ValueError("undeclared full configuration differences: " + ", ".join(sorted(undeclared)))
        unknown = [n for n, v in dims.items() if v["status"] == "unknown"]
        if unknown:
            raise ValueError("unknown training evidence dimensions: " + ", ".join(unknown))
        forbidden = [n for n, v in dims.items() if v["status"] == "different" and n not in allowed]
        if forbidden:
            raise ValueError("undeclared between-condition differences: " + ", ".join(forbidden))
        entry = {"seed": seed, "comparison": comparison, "full_configuration_differences": full}
        for side in ("left", "right"):
            report, path, report_sha = loaded[side]
            desc = report.get("training_descriptor", {})
            if type(desc.get("seed")) is not int or desc["seed"] != seed:
                raise ValueError("checkpoint descriptor seed differs from declared pair seed")
            if desc.get("completion_status") != "complete":
                raise ValueError("seed comparison requires complete training segments")
            for key in ("training_manifest_sha256", "validation_manifest_sha256", "target_plan_sha256",
                        "available_prefix_plan_sha256"):
                _hash(report.get(key), key)
            if type(report.get("evaluation_seed")) is not int or report["evaluation_seed"] < 0:
                raise ValueError("known nonnegative evaluation seed is required")
            signature = {k: report.get(k) for k in ("target_plan", "target_plan_sha256", "validation_manifest_sha256",
                                                     "training_manifest_sha256", "evaluation_seed", "context",
                                                     "available_prefix_plan_sha256")}
            if baseline is None:
                baseline = signature
            elif signature != baseline:
                raise ValueError("all seed reports require identical validation targets, context and prefixes")
            if side in references:
                ref = references[side]
                within = _differences(_configuration(ref, ref["training_descriptor"]["seed"]), configs[side],
                                      ignore_seed=True)
                if within:
                    raise ValueError("within-condition full configuration differs: " + ", ".join(within))
                same = _training_comparison(ref, report)["dimensions"]
                bad = [n for n, v in same.items() if n != "seed" and v["status"] != "matched"]
                if bad:
                    raise ValueError("within-condition training identity differs or is unknown: " + ", ".join(bad))
            else:
                references[side] = report
            shas = {"model": _hash(report.get("model_sha256"), "model_sha256"),
                    "state": _hash(report.get("checkpoint_state_sha256"), "checkpoint_state_sha256"),
                    "manifest": _hash(report.get("checkpoint_manifest_sha256"), "checkpoint_manifest_sha256")}
            for key, value in shas.items():
                if value in ids[side][key]:
                    if key != "model":
                        raise ValueError("duplicate checkpoint identity within condition")
                    dup_models[side].append({"seed": seed, "model_sha256": value})
                ids[side][key].add(value)
            entry[side] = {"report_path": path, "report_sha256": report_sha, "model_sha256": shas["model"],
                           "checkpoint_state_sha256": shas["state"], "checkpoint_manifest_sha256": shas["manifest"],
                           "checkpoint": report.get("checkpoint"), "training_descriptor": desc}
        per_seed.append(entry)
    cross = [{"identity": k, "sha256": sorted(ids["left"][k] & ids["right"][k])}
             for k in ("model", "state", "manifest") if ids["left"][k] & ids["right"][k]]
    deltas = [r["comparison"]["delta_ce_right_minus_left"] for r in per_seed]
    lce = [r["comparison"]["left"]["ce"] for r in per_seed]
    rce = [r["comparison"]["right"]["ce"] for r in per_seed]
    if not all(type(v) in (int, float) and math.isfinite(v) for v in deltas + lce + rce):
        raise ValueError("per-seed CE and deltas must be finite")
    n = len(per_seed)
    sd = statistics.stdev(deltas)
    se = abs(deltas[0] - deltas[1]) / 2 if n == 2 else sd / math.sqrt(n)
    tokens = per_seed[0]["comparison"]["prediction_tokens"]
    report = {"kind": "paired_seed_validation_comparison", "allowed_between_dimensions": list(allowed),
              "per_seed": per_seed,
              "aggregate": {"seeds": n, "mean_ce_left": statistics.mean(lce), "mean_ce_right": statistics.mean(rce),
                            "mean_paired_delta_ce": statistics.mean(deltas), "paired_delta_sample_sd": sd,
                            "paired_delta_standard_error": se,
                            "weighting": "equal weight per seed; each CE is token-weighted on identical targets"},
              "training_identity": {"left": references["left"]["training_descriptor"],
                                    "right": references["right"]["training_descriptor"]},
              "validation": {"manifest_sha256": baseline["validation_manifest_sha256"],
                             "target_plan_sha256": baseline["target_plan_sha256"], "context": baseline["context"],
                             "available_prefix_plan_sha256": baseline["available_prefix_plan_sha256"],
                             "unique_prediction_tokens": tokens, "repeated_prediction_tokens_per_condition": n * tokens,
                             "total_scored_prediction_tokens_across_conditions": 2 * n * tokens},
              "cross_condition_duplicate_identities": cross, "duplicate_model_outcomes": dup_models,
              "unique_model_count": {s: len(ids[s]["model"]) for s in ("left", "right")},
              "automatic_ranking_eligible": False,
              "uncertainty_scope": "sample SD/SE across seed-pair deltas; no seed interval or p-value; document "
                                   "intervals are not seed variance",
              "limitations": ["the same numeric seed does not establish coupled random streams",
                              "reports do not establish prospective declaration or absence of selection",
                              "checkpoint hashes are report-bound identities, not revalidated contents"]}
    _publish_json(out_dir, "replication.json", report)
    return report
