"""Memory-mapped per-split document index for the packed sampler (reference tnlm/sampler_index.py).

``<dataset>/.sampler-index-v1/<split>.index.bin`` holds one 40-byte record per document of the split
(int64 token_start, token_end, numeric_id, byte offset and length of its ``documents.jsonl`` line),
so samplers over large corpora touch only the rows they pack instead of parsing all metadata.
The index is derived data: it is verified against the manifest's documents.jsonl checksum and
rebuilt when missing or stale; several ranks may share it read-only.
"""
from __future__ import annotations

import fcntl
import hashlib
import json
import os
import tempfile
from collections.abc import Mapping, Sequence
from pathlib import Path

import numpy as np

from .token_format import SPLIT_ORDER

INDEX_DIR = ".sampler-index-v1"
RECORD = np.dtype([("token_start", "<i8"), ("token_end", "<i8"), ("numeric_id", "<i8"), ("offset", "<i8"),
                   ("length", "<i8")])


def _identity(manifest) -> dict:
    return {"version": 1, "documents_sha256": manifest["artifacts"]["documents.jsonl"]}


def _build(root: Path, manifest, cache: Path):
    per_split = {s: [] for s in SPLIT_ORDER}
    offset = 0
    with (root / "documents.jsonl").open("rb") as fh:
        for raw in fh:
            doc = json.loads(raw)
            per_split[doc["split"]].append((doc["token_start"], doc["token_end"], doc["numeric_id"], offset, len(raw)))
            offset += len(raw)
    cache.mkdir(exist_ok=True)
    for split, rows in per_split.items():
        arr = np.array(rows, dtype=RECORD) if rows else np.empty(0, dtype=RECORD)
        fd, tmp = tempfile.mkstemp(dir=cache, prefix=f".{split}-")
        with os.fdopen(fd, "wb") as out:
            out.write(arr.tobytes())
            out.flush()
            os.fsync(out.fileno())
        os.replace(tmp, cache / f"{split}.index.bin")
    meta = {"identity": _identity(manifest), "counts": {s: len(r) for s, r in per_split.items()}}
    fd, tmp = tempfile.mkstemp(dir=cache, prefix=".identity-")
    with os.fdopen(fd, "w") as out:
        json.dump(meta, out, sort_keys=True)
        out.flush()
        os.fsync(out.fileno())
    os.replace(tmp, cache / "identity.json")


def ensure_sampler_index(root, manifest, *, rebuild: bool = False) -> Path:
    root = Path(root)
    cache = root / INDEX_DIR
    cache.mkdir(exist_ok=True)
    with (cache / "build.lock").open("a") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        ok = False
        if not rebuild:
            try:
                meta = json.loads((cache / "identity.json").read_text())
                ok = meta["identity"] == _identity(manifest) and all(
                    (cache / f"{s}.index.bin").stat().st_size == meta["counts"][s] * RECORD.itemsize
                    for s in SPLIT_ORDER)
            except (OSError, ValueError, KeyError):
                ok = False
        if not ok:
            _build(root, manifest, cache)
    return cache


class _Document(Mapping):
    def __init__(self, owner, index):
        self._owner, self._index, self._doc = owner, index, None

    def _load(self):
        if self._doc is None:
            self._doc = self._owner.full_document(self._index)
        return self._doc

    def __getitem__(self, key):
        row = self._owner.rows[self._index]
        if key in ("token_start", "token_end", "numeric_id"):
            return int(row[key])
        return self._load()[key]

    def __iter__(self):
        return iter(self._load())

    def __len__(self):
        return len(self._load())


class IndexedDocuments(Sequence):
    """Documents of one split, in ``documents.jsonl`` order."""

    def __init__(self, root, cache, split):
        self.root, self.cache_dir, self.split = Path(root), Path(cache), split
        path = self.cache_dir / f"{split}.index.bin"
        n = path.stat().st_size // RECORD.itemsize
        self.rows = np.memmap(path, dtype=RECORD, mode="r", shape=(n,)) if n else np.empty(0, dtype=RECORD)
        self._meta = self.root / "documents.jsonl"

    def length(self, i):
        r = self.rows[i]
        return int(r["token_end"] - r["token_start"])

    def start(self, i):
        return int(self.rows[i]["token_start"])

    def numeric_id(self, i):
        return int(self.rows[i]["numeric_id"])

    def full_document(self, i):
        r = self.rows[i]
        with self._meta.open("rb") as fh:
            fh.seek(int(r["offset"]))
            return json.loads(fh.read(int(r["length"])))

    def __len__(self):
        return len(self.rows)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        return _Document(self, i)


def load_sampler_index(root, manifest, split, *, rebuild: bool = False) -> IndexedDocuments:
    if split not in SPLIT_ORDER:
        raise ValueError(f"invalid split: {split}")
    cache = ensure_sampler_index(root, manifest, rebuild=rebuild)
    return IndexedDocuments(root, cache, split)


def index_digest(root) -> str:
    """sha256 over the split index files (for cross-rank agreement checks)."""
    h = hashlib.sha256()
    cache = Path(root) / INDEX_DIR
    for s in SPLIT_ORDER:
        h.update((cache / f"{s}.index.bin").read_bytes())
    return h.hexdigest()
