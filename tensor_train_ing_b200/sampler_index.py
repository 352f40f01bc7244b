"""Memory-mapped per-split document index for the packed sampler (reference tnlm/sampler_index.py).

``<dataset>/.sampler-index-v1/<split>.index.bin`` holds one 40-byte record per document of the split
(int64 token_start, token_end, numeric_id, byte offset and length of its ``documents.jsonl`` line),
so samplers over large corpora touch only the rows they pack instead of parsing all metadata.
``index.json`` beside them records the source identity (sha256 of the canonical manifest and of
documents.jsonl), the row layout and each split's count, size and sha256.  Directory, files, rows
and header are the reference platform's, so either framework reads an index the other built.  The
index is derived data: it is verified on load and rebuilt when missing or stale (the reference
instead asks for an explicit rebuild); builds take the dataset's ``.sampler-index-v1.lock``.

A long run reads rows from all over the index (one epoch visits every document in shuffled order),
so without a bound the mapping's resident pages would grow to the whole file.  ``IndexedDocuments``
counts its row reads and, every ``RELEASE_EVERY`` of them, drops this process's resident pages of the
mapping with ``madvise(MADV_DONTNEED)`` (reference ``tnlm/sampler_index.py:247-320`` bounds residency
the same way).  The file is read-only and shared, so a release changes no value: later reads fault
the pages back in from the page cache.
"""
from __future__ import annotations

import fcntl
import hashlib
import json
import mmap
import os
import tempfile
from collections.abc import Mapping, Sequence
from pathlib import Path

import numpy as np

from .token_format import SPLIT_ORDER

INDEX_DIR = ".sampler-index-v1"
RECORD = np.dtype([("token_start", "<i8"), ("token_end", "<i8"), ("numeric_id", "<i8"),
                   ("metadata_offset", "<i8"), ("metadata_length", "<i8")])
INDEX_VERSION = 1


def _identity(manifest) -> dict:
    """The manifest's canonical text is what ``manifest.json`` holds once published (and what
    ``manifest.sha256`` covers), so the identity is the same before and after publication."""
    canonical = json.dumps(manifest, sort_keys=True, indent=2) + "\n"
    return {"manifest_sha256": hashlib.sha256(canonical.encode("utf-8")).hexdigest(),
            "documents_sha256": manifest["artifacts"]["documents.jsonl"]}


def _file_sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as fh:
        for block in iter(lambda: fh.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _write_atomic(path: Path, data: bytes):
    fd, tmp = tempfile.mkstemp(dir=path.parent, prefix=f".{path.name}-")
    with os.fdopen(fd, "wb") as out:
        out.write(data)
        out.flush()
        os.fsync(out.fileno())
    os.replace(tmp, path)


def _build(root: Path, manifest, cache: Path):
    per_split = {s: [] for s in SPLIT_ORDER}
    offset = 0
    with (root / "documents.jsonl").open("rb") as fh:
        for raw in fh:
            doc = json.loads(raw)
            per_split[doc["split"]].append((doc["token_start"], doc["token_end"], doc["numeric_id"], offset, len(raw)))
            offset += len(raw)
    cache.mkdir(exist_ok=True)
    splits = {}
    for split, rows in per_split.items():
        arr = np.array(rows, dtype=RECORD) if rows else np.empty(0, dtype=RECORD)
        _write_atomic(cache / f"{split}.index.bin", arr.tobytes())
        splits[split] = {"count": len(rows), "bytes": arr.nbytes, "sha256": _file_sha256(cache / f"{split}.index.bin")}
    header = {"index_version": INDEX_VERSION, "identity": _identity(manifest), "row_bytes": RECORD.itemsize,
              "fields": list(RECORD.names), "splits": splits}
    _write_atomic(cache / "index.json", (json.dumps(header, sort_keys=True, indent=2) + "\n").encode("utf-8"))
    (cache / "identity.json").unlink(missing_ok=True)  # header of an earlier layout


def _valid(cache: Path, manifest) -> bool:
    try:
        header = json.loads((cache / "index.json").read_text())
        if (header["index_version"] != INDEX_VERSION or header["identity"] != _identity(manifest)
                or header["row_bytes"] != RECORD.itemsize or header["fields"] != list(RECORD.names)
                or set(header["splits"]) != set(SPLIT_ORDER)):
            return False
        for split in SPLIT_ORDER:
            info, path = header["splits"][split], cache / f"{split}.index.bin"
            if (info["bytes"] != info["count"] * RECORD.itemsize or path.stat().st_size != info["bytes"]
                    or _file_sha256(path) != info["sha256"]):
                return False
        return True
    except (OSError, ValueError, KeyError, TypeError):
        return False


def ensure_sampler_index(root, manifest, *, rebuild: bool = False) -> Path:
    root = Path(root)
    cache = root / INDEX_DIR
    with (root / f"{INDEX_DIR}.lock").open("a+b") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if rebuild or not _valid(cache, manifest):
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
    """Documents of one split, in ``documents.jsonl`` order.

    ``length``, ``start``, ``numeric_id`` and item access read one index row each; every
    ``RELEASE_EVERY`` such reads the mapping's resident pages are released (``release_pages``).
    Code that reads ``rows`` directly bypasses the count and may call ``release_pages`` itself."""

    RELEASE_EVERY = 4096

    def __init__(self, root, cache, split):
        self.root, self.cache_dir, self.split = Path(root), Path(cache), split
        path = self.cache_dir / f"{split}.index.bin"
        n = path.stat().st_size // RECORD.itemsize
        self.rows = np.memmap(path, dtype=RECORD, mode="r", shape=(n,)) if n else np.empty(0, dtype=RECORD)
        self._meta = (self.root / "documents.jsonl").open("rb")
        self.reads = 0         # row reads since the last release
        self.releases = 0      # releases that took effect

    def release_pages(self) -> bool:
        """Drop this process's resident pages of the index mapping.  False where the platform has no
        ``madvise``/``MADV_DONTNEED`` or the call fails (the values read are the same either way)."""
        self.reads = 0
        mapped = getattr(self.rows, "_mmap", None)
        advice = getattr(mmap, "MADV_DONTNEED", None)
        if mapped is None or advice is None or not hasattr(mapped, "madvise"):
            return False
        try:
            mapped.madvise(advice)
        except (OSError, ValueError):
            return False
        self.releases += 1
        return True

    def _row(self, i):
        n = len(self.rows)
        i = int(i)
        if i < 0:
            i += n
        if not 0 <= i < n:
            raise IndexError(f"document {i} outside a split of {n}")
        self.reads += 1
        if self.reads >= self.RELEASE_EVERY:
            self.release_pages()
        return i, self.rows[i]

    def length(self, i):
        _, r = self._row(i)
        return int(r["token_end"] - r["token_start"])

    def start(self, i):
        return int(self._row(i)[1]["token_start"])

    def numeric_id(self, i):
        return int(self._row(i)[1]["numeric_id"])

    def full_document(self, i):
        _, r = self._row(i)
        raw = os.pread(self._meta.fileno(), int(r["metadata_length"]), int(r["metadata_offset"]))
        return json.loads(raw)

    def close(self):
        self._meta.close()

    def __len__(self):
        return len(self.rows)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        return _Document(self, self._row(i)[0])


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
