"""Compare several pairs of held-out evaluation reports and publish them as one bundle.

Every pair is checked and compared before anything is written; then ``comparisons.json`` appears in
a new directory in one durable write.  A report named by several pairs is read once, and the bundle
binds each input path to the sha256 and size of the exact bytes compared.  Each result is what
``evaluate.compare_evaluations`` returns for the pair (with its paired document bootstrap); the
bundle adds no pooled estimate, ranking or multiplicity correction.  Same contract as the
reference's batch comparator (tnlm/comparison_batch.py:12-68).
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

from .durable import new_dir_with_json
from .evaluate import compare_evaluations

MAX_BOOTSTRAP = 100_000


class ReportStore:
    """Evaluation reports by resolved path, each read and fingerprinted once."""

    def __init__(self):
        self.by_path: dict[str, dict] = {}
        self.fingerprints: dict[str, dict] = {}

    def load(self, where) -> tuple[str, dict, str]:
        """(resolved path, report, sha256 of its bytes)."""
        if not isinstance(where, (str, Path)):
            raise ValueError(f"a report input must be a path, not {type(where).__name__}")
        path = str(Path(where).resolve())
        if path not in self.by_path:
            blob = Path(path).read_bytes()
            report = json.loads(blob)
            if not isinstance(report, dict):
                raise ValueError(f"{path} does not hold a JSON object")
            self.by_path[path] = report
            self.fingerprints[path] = {"sha256": hashlib.sha256(blob).hexdigest(), "bytes": len(blob)}
        return path, self.by_path[path], self.fingerprints[path]["sha256"]


def compare_evaluation_pairs(pairs, out_dir, *, bootstrap_samples=1000, seed=0):
    """``pairs``: ordered ``{"name", "left", "right"}`` mappings with unique nonempty names."""
    if not isinstance(pairs, list) or not pairs:
        raise ValueError("a comparison batch needs a nonempty list of pairs")
    if type(bootstrap_samples) is not int or not 0 <= bootstrap_samples <= MAX_BOOTSTRAP:
        raise ValueError(f"bootstrap_samples must be an integer in [0, {MAX_BOOTSTRAP}]")
    if type(seed) is not int or seed < 0:
        raise ValueError("the bootstrap seed must be a nonnegative integer")
    reports = ReportStore()
    used, results = set(), []
    for pair in pairs:
        if not isinstance(pair, dict) or set(pair) != {"name", "left", "right"}:
            raise ValueError("a comparison pair is a mapping with exactly the keys name, left and right")
        label = pair["name"]
        if not isinstance(label, str) or not label.strip() or label in used:
            raise ValueError(f"comparison name {label!r} is empty or used twice")
        used.add(label)
        lpath, left, _ = reports.load(pair["left"])
        rpath, right, _ = reports.load(pair["right"])
        outcome = compare_evaluations(left, right, None, bootstrap_samples=bootstrap_samples, seed=seed)
        results.append({"name": label, "left": lpath, "right": rpath, "result": outcome})
    bundle = {"kind": "batched_validation_comparisons", "pairs": results, "inputs": reports.fingerprints,
              "bootstrap_samples": bootstrap_samples, "seed": seed, "automatic_ranking_eligible": False,
              "scope": "each pair compared on its own matched targets; intervals are paired document "
                       "bootstraps, not training-seed variance; no pooled estimate, ranking or "
                       "multiplicity correction"}
    new_dir_with_json(out_dir, "comparisons.json", bundle)
    return bundle
