"""Export one sweep candidate's recorded configuration as YAML that ``tnlm train`` accepts.

The sweep journal (``sweep.json``, written by sweep.py) freezes an identity record and stores its
canonical sha256 beside it; every trajectory inside carries its configuration and that
configuration's canonical sha256.  The export re-derives both digests, so a journal edited after
it was written is refused, and writes the saved values verbatim: defaults of the current schema are
not filled in.  Behaviour as the reference's exporter (tnlm/sweep_config.py:14-44).
"""
from __future__ import annotations

import json
from pathlib import Path

import yaml

from .hashing import canonical_sha256, file_sha256

_JOURNAL = "sweep.json"


def _identity(journal: dict) -> dict:
    identity = journal.get("identity")
    if not isinstance(identity, dict) or identity.get("version") != 1:
        raise ValueError("the sweep journal has no identity record of a supported version")
    if canonical_sha256(identity) != journal.get("identity_sha256"):
        raise ValueError("the sweep identity does not match its recorded sha256")
    rows = identity.get("trajectories")
    if not isinstance(rows, list) or any(not isinstance(r, dict) for r in rows):
        raise ValueError("the sweep identity's trajectory list is malformed")
    return identity


def _trajectory(identity: dict, name: str) -> dict:
    hits = [r for r in identity["trajectories"] if r.get("name") == name]
    if len(hits) != 1:
        raise ValueError(f"{len(hits)} recorded trajectories are named {name!r}; exactly one is needed")
    row = hits[0]
    config = row.get("config")
    if not (isinstance(config, dict) and isinstance(config.get("model"), dict) and isinstance(config.get("train"), dict)):
        raise ValueError(f"trajectory {name!r} has no model and train configuration")
    if canonical_sha256(config) != row.get("config_sha256"):
        raise ValueError(f"trajectory {name!r}'s configuration does not match its recorded sha256")
    return row


def export_sweep_config(sweep, candidate) -> str:
    path = Path(sweep) / _JOURNAL
    journal = json.loads(path.read_bytes())
    identity = _identity(journal)
    row = _trajectory(identity, candidate)
    provenance = {"source": str(path.resolve()), "source_sha256": file_sha256(path), "candidate": candidate,
                  "identity_sha256": journal["identity_sha256"], "config_sha256": row["config_sha256"]}
    header = ["# Configuration exactly as the sweep recorded it (no schema defaults added).",
              "# Exporting it says nothing about whether the candidate's checkpoints completed.",
              "# provenance: " + json.dumps(provenance, sort_keys=True)]
    return "\n".join(header) + "\n" + yaml.safe_dump(row["config"], sort_keys=False)
