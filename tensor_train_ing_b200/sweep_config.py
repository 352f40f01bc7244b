"""Export one recorded sweep candidate's exact configuration as YAML (reference tnlm/sweep_config.py)."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import yaml


def _digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()).hexdigest()


def export_sweep_config(sweep, candidate) -> str:
    """YAML of the candidate's saved configuration (no current defaults injected), with a provenance
    comment binding it to the sweep journal's bytes and identity checksum."""
    path = Path(sweep) / "sweep.json"
    raw = path.read_bytes()
    journal = json.loads(raw)
    identity = journal.get("identity")
    if not isinstance(identity, dict) or identity.get("version") != 1:
        raise ValueError("unsupported or missing sweep identity")
    if _digest(identity) != journal.get("identity_sha256"):
        raise ValueError("sweep identity checksum mismatch")
    rows = identity.get("trajectories")
    if not isinstance(rows, list) or not all(isinstance(r, dict) for r in rows):
        raise ValueError("invalid sweep trajectories")
    chosen = [r for r in rows if r.get("name") == candidate]
    if len(chosen) != 1:
        raise ValueError("candidate must match exactly one recorded trajectory")
    config = chosen[0].get("config")
    if not isinstance(config, dict) or not all(isinstance(config.get(k), dict) for k in ("model", "train")):
        raise ValueError("invalid recorded candidate configuration")
    if _digest(config) != chosen[0].get("config_sha256"):
        raise ValueError("candidate config checksum mismatch")
    provenance = {"source": str(path.resolve()), "source_sha256": hashlib.sha256(raw).hexdigest(),
                  "candidate": candidate, "identity_sha256": journal["identity_sha256"],
                  "config_sha256": chosen[0]["config_sha256"]}
    return ("# Exact recorded sweep config; current schema defaults are not injected.\n"
            "# This export does not certify checkpoint completion.\n"
            "# provenance: " + json.dumps(provenance, sort_keys=True) + "\n" + yaml.safe_dump(config, sort_keys=False))
