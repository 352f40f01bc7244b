"""Paired-seed replication summaries built from evaluation reports (no model runs).

Each ``{seed, left, right}`` pair names two evaluation reports: condition "left" and condition
"right", both trained with that seed and scored on the same frozen validation targets.  The summary
is the equal-weight mean over seeds of the per-seed CE difference (right minus left) with its sample
SD and standard error; no confidence interval, p-value or winner is drawn.  The checks and the
report schema follow the reference's comparator (tnlm/replication.py:61-225):

* between the conditions, every difference in the training descriptors or in the full recorded
  configurations must be declared in ``allowed_between_dimensions`` (descriptor dimension names,
  which also cover their configuration paths, or ``config.*`` paths); the seed never may;
* within a condition, the recorded configurations agree on everything but ``train.seed`` and the
  training descriptors match in every dimension but the seed;
* every report scores the same targets (plan, manifests, evaluation seed, context, prefix plan);
* checkpoint state and manifest digests are unique within a condition; a repeated model digest is
  allowed but listed, and digests shared across the conditions are listed too.

Every check runs before the output directory is created.
"""
from __future__ import annotations

import math
import statistics

from .comparison_batch import ReportStore
from .durable import new_dir_with_json
from .evaluate import _training_comparison, compare_evaluations

SIDES = ("left", "right")
IDENTITIES = (("model", "model_sha256"), ("state", "checkpoint_state_sha256"),
              ("manifest", "checkpoint_manifest_sha256"))
TARGET_FIELDS = ("target_plan", "target_plan_sha256", "validation_manifest_sha256", "training_manifest_sha256",
                 "evaluation_seed", "context", "available_prefix_plan_sha256")

# descriptor dimension -> the configuration path a declared difference in it also covers
_DIMENSION_PATHS = {
    "optimizer": "train.optimizer", "width": "model.d_model", "depth": "model.layers",
    "train_context": "data.context", "rung_total_tokens": "train.rung_total_tokens",
    "global_prediction_tokens_per_update": "train.global_prediction_tokens_per_update", "lr": "train.lr",
    "normalization": "model.normalization", "attention": "model.attention", "aux_adamw_lr": "train.aux_adamw_lr",
    "schedule": "train.schedule",
}
_DIMENSION_PATHS.update({k: "model." + k for k in (
    "width_scaling_base", "width_lr_exponent", "width_logit_exponent", "depth_scaling_base", "depth_lr_exponent",
    "depth_residual_base", "depth_residual_exponent", "residual_alpha")})
_DIMENSION_PATHS.update({k: "train." + k for k in ("weight_decay_hidden", "beta1", "beta2")})


def _sha(value, what: str) -> str:
    if not (isinstance(value, str) and len(value) == 64 and set(value) <= set("0123456789abcdef")):
        raise ValueError(f"{what} is not a sha256 hex digest")
    return value


def flatten_config(tree, root: str = "config") -> dict:
    """Dot-path leaves of a configuration mapping (an empty mapping is kept as a leaf)."""
    leaves, stack = {}, [(root, tree)]
    while stack:
        path, node = stack.pop()
        if not isinstance(node, dict):
            leaves[path] = node
            continue
        if not node:
            leaves[path] = {}
        for key, child in node.items():
            if not isinstance(key, str) or "." in key:
                raise ValueError(f"configuration key {key!r} under {path} cannot be a dot-path component")
            stack.append((f"{path}.{key}", child))
    return leaves


def config_differences(a: dict, b: dict, *, ignore: tuple = ()) -> list[str]:
    fa, fb = flatten_config(a), flatten_config(b)
    if fa.keys() != fb.keys():
        raise ValueError("the two recorded configurations do not have the same set of fields")
    return sorted(k for k in fa if k not in ignore and (type(fa[k]) is not type(fb[k]) or fa[k] != fb[k]))


def _recorded_config(report: dict, seed: int) -> dict:
    cfg = report.get("training_descriptor", {}).get("configuration")
    ok = (isinstance(cfg, dict) and isinstance(cfg.get("model"), dict) and isinstance(cfg.get("train"), dict)
          and "project" not in cfg and type(cfg["train"].get("seed")) is int and cfg["train"]["seed"] == seed)
    if not ok:
        raise ValueError(f"seed {seed}: the report lacks a complete recorded configuration with that seed")
    return cfg


class _Condition:
    """One side's reports across seeds: its first report is the within-condition reference."""

    def __init__(self, side: str):
        self.side = side
        self.first: dict | None = None
        self.seen = {name: set() for name, _ in IDENTITIES}
        self.repeated_models: list[dict] = []

    def admit(self, seed: int, report: dict, path: str, report_sha: str, cfg: dict) -> dict:
        desc = report.get("training_descriptor", {})
        if type(desc.get("seed")) is not int or desc["seed"] != seed:
            raise ValueError(f"seed {seed}: the {self.side} checkpoint was trained with another seed")
        if desc.get("completion_status") != "complete":
            raise ValueError(f"seed {seed}: the {self.side} training segment is not complete")
        if self.first is None:
            self.first = report
        else:
            ref_cfg = _recorded_config(self.first, self.first["training_descriptor"]["seed"])
            drift = config_differences(ref_cfg, cfg, ignore=("config.train.seed",))
            if drift:
                raise ValueError(f"{self.side} condition: configurations differ across seeds in " + ", ".join(drift))
            dims = _training_comparison(self.first, report)["dimensions"]
            off = [n for n, v in dims.items() if n != "seed" and v["status"] != "matched"]
            if off:
                raise ValueError(f"{self.side} condition: training identity differs or is unknown in "
                                 + ", ".join(off))
        digests = {}
        for name, key in IDENTITIES:
            digest = _sha(report.get(key), key)
            if digest in self.seen[name]:
                if name != "model":
                    raise ValueError(f"{self.side} condition: two seeds share one checkpoint {name} digest")
                self.repeated_models.append({"seed": seed, "model_sha256": digest})
            self.seen[name].add(digest)
            digests[key] = digest
        return {"report_path": path, "report_sha256": report_sha, **digests,
                "checkpoint": report.get("checkpoint"), "training_descriptor": desc}


def _check_between(seed: int, comparison: dict, cfgs: dict, allowed: list) -> list[str]:
    dims = comparison["training_comparison"]["dimensions"]
    paths = flatten_config(cfgs["left"]).keys() & flatten_config(cfgs["right"]).keys()
    strangers = [a for a in allowed if a not in dims and a not in paths]
    if strangers:
        raise ValueError("allowed_between_dimensions names unknown dimensions or paths: " + ", ".join(strangers))
    full = config_differences(cfgs["left"], cfgs["right"])
    covered = set(allowed) | {"config." + _DIMENSION_PATHS[a] for a in allowed if a in _DIMENSION_PATHS}
    undeclared = sorted(set(full) - covered)
    if undeclared:
        raise ValueError(f"seed {seed}: undeclared configuration differences: " + ", ".join(undeclared))
    unknown = [n for n, v in dims.items() if v["status"] == "unknown"]
    if unknown:
        raise ValueError(f"seed {seed}: training evidence unknown for " + ", ".join(unknown))
    extra = [n for n, v in dims.items() if v["status"] == "different" and n not in allowed]
    if extra:
        raise ValueError(f"seed {seed}: undeclared between-condition differences: " + ", ".join(extra))
    return full


def _target_signature(report: dict, seed: int) -> dict:
    for key in ("training_manifest_sha256", "validation_manifest_sha256", "target_plan_sha256",
                "available_prefix_plan_sha256"):
        _sha(report.get(key), key)
    if type(report.get("evaluation_seed")) is not int or report["evaluation_seed"] < 0:
        raise ValueError(f"seed {seed}: the report has no nonnegative evaluation seed")
    return {k: report.get(k) for k in TARGET_FIELDS}


def _aggregate(rows: list[dict]) -> dict:
    deltas = [r["comparison"]["delta_ce_right_minus_left"] for r in rows]
    left = [r["comparison"]["left"]["ce"] for r in rows]
    right = [r["comparison"]["right"]["ce"] for r in rows]
    if not all(type(v) in (int, float) and math.isfinite(v) for v in deltas + left + right):
        raise ValueError("a per-seed CE or CE difference is not finite")
    sd = statistics.stdev(deltas)
    # two seeds: half the spread of the two differences; more: the usual SD / sqrt(n)
    se = abs(deltas[0] - deltas[1]) / 2 if len(rows) == 2 else sd / math.sqrt(len(rows))
    return {"seeds": len(rows), "mean_ce_left": statistics.mean(left), "mean_ce_right": statistics.mean(right),
            "mean_paired_delta_ce": statistics.mean(deltas), "paired_delta_sample_sd": sd,
            "paired_delta_standard_error": se,
            "weighting": "every seed weighs the same; each CE is token-weighted over the same targets"}


def compare_seed_pairs(pairs, out_dir, *, allowed_between_dimensions) -> dict:
    if not isinstance(pairs, list) or len(pairs) < 2:
        raise ValueError("a replication summary needs at least two seed pairs")
    allowed = allowed_between_dimensions
    if (not isinstance(allowed, list) or not all(isinstance(a, str) for a in allowed)
            or len(set(allowed)) != len(allowed)):
        raise ValueError("allowed_between_dimensions must be a list of unique names")
    if {"seed", "config.train.seed"} & set(allowed):
        raise ValueError("the seed cannot be an allowed between-condition difference")
    store = ReportStore()
    conditions = {s: _Condition(s) for s in SIDES}
    seeds, rows, signature = set(), [], None
    for pair in pairs:
        if not isinstance(pair, dict) or set(pair) != {"seed", "left", "right"}:
            raise ValueError("a seed pair is a mapping with exactly seed, left and right")
        seed = pair["seed"]
        if type(seed) is not int or seed < 0 or seed in seeds:
            raise ValueError(f"pair seed {seed!r} must be one of unique nonnegative integers")
        seeds.add(seed)
        loaded = {s: store.load(pair[s]) for s in SIDES}
        reports = {s: loaded[s][1] for s in SIDES}
        comparison = compare_evaluations(reports["left"], reports["right"], None, bootstrap_samples=0)
        cfgs = {s: _recorded_config(reports[s], seed) for s in SIDES}
        row = {"seed": seed, "comparison": comparison,
               "full_configuration_differences": _check_between(seed, comparison, cfgs, allowed)}
        for s in SIDES:
            sig = _target_signature(reports[s], seed)
            if signature is None:
                signature = sig
            elif sig != signature:
                raise ValueError(f"seed {seed}: the {s} report scores other validation targets, context or prefixes")
            path, report, sha = loaded[s]
            row[s] = conditions[s].admit(seed, report, path, sha, cfgs[s])
        rows.append(row)
    shared = []
    for name, _ in IDENTITIES:
        both = conditions["left"].seen[name] & conditions["right"].seen[name]
        if both:
            shared.append({"identity": name, "sha256": sorted(both)})
    tokens = rows[0]["comparison"]["prediction_tokens"]
    summary = {
        "kind": "paired_seed_validation_comparison", "allowed_between_dimensions": list(allowed),
        "per_seed": rows, "aggregate": _aggregate(rows),
        "training_identity": {"left": conditions["left"].first["training_descriptor"],
                              "right": conditions["right"].first["training_descriptor"],
                              "reference_seed_scope": "the first pair's descriptors stand for the dimensions "
                                                      "every seed matches; seeds differ"},
        "validation": {"manifest_sha256": signature["validation_manifest_sha256"],
                       "target_plan_sha256": signature["target_plan_sha256"], "context": signature["context"],
                       "available_prefix_plan_sha256": signature["available_prefix_plan_sha256"],
                       "unique_prediction_tokens": tokens,
                       "repeated_prediction_tokens_per_condition": len(rows) * tokens,
                       "total_scored_prediction_tokens_across_conditions": 2 * len(rows) * tokens,
                       "scope": "one frozen validation target set scored once per checkpoint; scoring it again "
                                "adds no new targets"},
        "cross_condition_duplicate_identities": shared,
        "duplicate_model_outcomes": {s: conditions[s].repeated_models for s in SIDES},
        "unique_model_count": {s: len(conditions[s].seen["model"]) for s in SIDES},
        "configuration_identity_scope": "every recorded configuration section except project; across seeds only "
                                        "train.seed differs; every between-condition difference is declared",
        "automatic_ranking_eligible": False,
        "uncertainty_scope": "sample SD and standard error over the per-seed differences; no interval or "
                             "p-value over seeds; document bootstrap intervals are not seed variance",
        "limitations": ["one numeric seed does not make the two conditions' random streams coupled",
                        "the reports cannot show that the comparison was declared in advance, that runs were "
                        "independent, or that no selection over hyperparameters took place",
                        "checkpoint digests are the ones the reports carry; checkpoint contents are not re-read",
                        "equal configurations do not prove equal code or runtime; each comparison keeps the "
                        "source evidence its reports recorded",
                        "complete means the declared training segment finished; nothing is ranked or promoted"],
    }
    new_dir_with_json(out_dir, "replication.json", summary)
    return summary
