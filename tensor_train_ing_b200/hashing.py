"""Digests used for identities across the framework.

Configurations, sweep identities and ledger rows are identified by the sha256 of their canonical
JSON text (keys sorted, no whitespace, NaN and infinities refused), so the same values give the
same digest in every process and in the reference's tools, which use the same canonical form.
Files (checkpoint payloads, dataset splits) are identified by the sha256 of their bytes.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

_CHUNK = 1 << 22  # file digests read 4 MiB at a time


def canonical_json(value) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def canonical_sha256(value) -> str:
    return hashlib.sha256(canonical_json(value).encode()).hexdigest()


def text_sha256(text: str) -> str:
    return hashlib.sha256(text.encode()).hexdigest()


def file_sha256(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as fh:
        for block in iter(lambda: fh.read(_CHUNK), b""):
            h.update(block)
    return h.hexdigest()
