"""Immutable token datasets and the deterministic packed-row sampler.

Dataset layout (identical to the reference platform, tnlm/data.py:149-460, so datasets are shared):
``manifest.json`` (format_version 1; source, tokenizer, split fractions, token counts, artifact
sha256s), ``manifest.sha256``, ``documents.jsonl`` (one record per document: id, numeric_id, split,
hashes, source offset, token_start/token_end in its split file, ...), and
``{train,val,test,calibration}.tokens.bin`` (int32 LE, every document followed by EOS 50256).

Packing (tnlm/data.py:463-973, ``document-shuffle-row-overlap-incremental-v2``): each epoch
shuffles documents with ``random.Random(f"{seed}:{epoch}")``; rows of ``context + 1`` tokens are
filled document by document; when a document continues into the next row the last token of a row
is repeated as the first of the next (so every target is predicted once); targets never cross
documents (-100); short rows are padded with token 50256 and unique negative document ids.
The sampler's state dict and its resume/context-fork rules are the reference's.
"""
from __future__ import annotations

import copy
import hashlib
import json
import math
import os
import random
import shutil
from bisect import bisect_left
from pathlib import Path

import numpy as np
import torch

from .token_format import SPLIT_ORDER, TOKEN_DTYPE, read_split_tokens

PACKING_VERSION = "document-shuffle-row-overlap-incremental-v2"
EOS = 50256
GPT2_VOCAB = 50257


def _sha(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for block in iter(lambda: fh.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _digest(text: str) -> str:
    return hashlib.sha256(text.encode("utf-8")).hexdigest()


def _manifest_path(path) -> Path:
    path = Path(path)
    return path / "manifest.json" if path.is_dir() else path


def manifest_hash(path) -> str:
    """sha256 of a completed manifest, checked against its independently stored digest."""
    path = _manifest_path(path)
    digest = _sha(path)
    if path.with_name("manifest.sha256").read_text().strip() != digest:
        raise ValueError("manifest checksum mismatch")
    return digest


def validate_tokenizer_compatibility(training_manifest, validation_manifest, *, allow_test_only=False) -> dict:
    """Both datasets must declare the same tokenizer (production fingerprint, or identical
    metadata for explicitly allowed test-only fixtures)."""
    records, hashes = [], []
    for source in (training_manifest, validation_manifest):
        path = _manifest_path(source)
        hashes.append(manifest_hash(path))
        record = json.loads(path.read_text()).get("tokenizer")
        if not isinstance(record, dict):
            raise ValueError("dataset manifest lacks tokenizer metadata")
        records.append(record)
    left, right = records
    if left.get("test_only") or right.get("test_only"):
        if not allow_test_only:
            raise ValueError("test-only tokenizer manifests are not allowed here")
        if left != right:
            raise ValueError("tokenizer metadata mismatch between training and validation data")
        return {"kind": "test_only_metadata_equality", "manifest_hashes": hashes}
    fp = left.get("fingerprint_sha256")
    if not isinstance(fp, str) or fp != right.get("fingerprint_sha256"):
        raise ValueError("tokenizer fingerprint mismatch between training and validation data")
    return {"kind": "fingerprint", "fingerprint_sha256": fp, "manifest_hashes": hashes}


# ------------------------------------------------------------------------------------------ preparation
def _tokenizer_metadata(tokenizer):
    if tokenizer is not None:
        return tokenizer, {"name": getattr(tokenizer, "name", type(tokenizer).__name__), "injected": True,
                           "test_only": True, "eos_id": tokenizer.eot_token}
    import tiktoken  # the production tokenizer (GPT-2 BPE)
    tok = tiktoken.get_encoding("gpt2")
    ranks = sorted((k.hex(), v) for k, v in tok._mergeable_ranks.items())
    meta = {"name": "gpt2", "package": "tiktoken", "eos_id": tok.eot_token,
            "vocabulary_sha256": _digest(json.dumps(ranks)), "special_tokens": tok._special_tokens,
            "regex_pattern": tok._pat_str}
    meta["fingerprint_sha256"] = _digest(json.dumps({"ranks": ranks, "regex_pattern": tok._pat_str,
                                                     "special_tokens": tok._special_tokens}, sort_keys=True))
    return tok, meta


def _records_jsonl(path):
    with Path(path).open() as fh:
        for line_no, line in enumerate(fh, 1):
            if line.strip():
                yield json.loads(line), line_no


def _records_parquet(shards):
    import pyarrow.parquet as pq
    for shard, path in shards:
        pf = pq.ParquetFile(path)
        cols = [c for c in ("text", "id", "doc_id") if c in pf.schema_arrow.names]
        row = 0
        for batch in pf.iter_batches(batch_size=256, columns=cols):
            for rec in batch.to_pylist():
                yield rec, {"shard": shard, "row": row}
                row += 1


def _heldout_keys(manifest) -> set:
    path = _manifest_path(manifest)
    manifest_hash(path)
    info = json.loads(path.read_text())
    docs = path.with_name("documents.jsonl")
    if _sha(docs) != info.get("artifacts", {}).get("documents.jsonl"):
        raise ValueError("heldout documents artifact checksum mismatch")
    keys = set()
    with docs.open() as fh:
        for line in fh:
            row = json.loads(line)
            if row.get("split") == "val":
                keys.update({("id", row["id"]), ("raw", row["content_sha256"]),
                             ("processed", row["processed_sha256"])})
    if not keys:
        raise ValueError("heldout manifest has no validation documents")
    return keys


def prepare_data(output_dir, *, source_jsonl=None, revision, max_tokens=50_000_000, max_documents=100_000,
                 tokenizer=None, split_fractions=None, hf_dataset=None, hf_config=None, hf_data_files=None,
                 hf_shard_checksums=None, hf_local_shards=None, workers=1, tokenization_batch_bytes=1 << 20,
                 exclude_validation_manifest=None, on_shard_scanned=None):
    """Freeze a bounded, deduplicated, tokenized document set into an immutable dataset directory.

    Selection keeps the ``max_documents`` documents with the smallest sha256("selection\\0" + id)
    rank, tokenizes them in rank order up to ``max_tokens`` and assigns each to a split by
    sha256(id) against cumulative split fractions.  The output directory must not exist; it is
    removed again if preparation fails.  Returns the manifest path.
    """
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=False)
    try:
        return _prepare(out, source_jsonl, revision, max_tokens, max_documents, tokenizer, split_fractions,
                        hf_dataset, hf_config, hf_data_files, hf_shard_checksums, hf_local_shards,
                        exclude_validation_manifest, on_shard_scanned, workers, tokenization_batch_bytes)
    except BaseException:
        shutil.rmtree(out)
        raise


def _prepare(out, source_jsonl, revision, max_tokens, max_documents, tokenizer, split_fractions, hf_dataset,
             hf_config, hf_data_files, hf_shard_checksums, hf_local_shards, exclude_validation_manifest,
             on_shard_scanned, workers=1, tokenization_batch_bytes=1 << 20):
    if not revision or revision in ("main", "master", "latest"):
        raise ValueError("an immutable source revision is required")
    if any(type(v) is not int or v <= 0 for v in (max_tokens, max_documents)):
        raise ValueError("positive integer data bounds required")
    if (source_jsonl is None) == (hf_dataset is None):
        raise ValueError("specify exactly one local JSONL or HF dataset")
    fractions = split_fractions or {"train": .97, "val": .01, "test": .01, "calibration": .01}
    if set(fractions) != set(SPLIT_ORDER) or any(not math.isfinite(v) or v < 0 for v in fractions.values()) \
            or abs(sum(fractions.values()) - 1) > 1e-9:
        raise ValueError("split fractions must specify train/val/test/calibration and sum to one")
    fractions = {s: fractions[s] for s in SPLIT_ORDER}
    tok, tok_meta = _tokenizer_metadata(tokenizer)
    if tok.eot_token != EOS:
        raise ValueError("GPT2 EOS must be 50256")
    if source_jsonl is not None:
        src = Path(source_jsonl).resolve()
        source = {"kind": "jsonl", "revision": revision, "path": str(src), "sha256": _sha(src)}
        records = _records_jsonl(src)
    else:
        if len(revision) != 40 or not hf_data_files or hf_local_shards is None:
            raise ValueError("HF mode needs a full 40-character commit, explicit data_files and local shard paths "
                             "(this machine has no network)")
        shards = [hf_data_files] if isinstance(hf_data_files, str) else list(hf_data_files)
        if not isinstance(hf_shard_checksums, dict) or set(hf_shard_checksums) != set(shards):
            raise ValueError("HF shard_checksums must cover every explicit shard exactly")
        verified = []
        for shard in sorted(shards):
            path = Path(hf_local_shards[shard])
            if _sha(path) != hf_shard_checksums[shard].lower():
                raise ValueError(f"HF raw shard checksum mismatch: {shard}")
            verified.append((shard, path))
        source = {"kind": "huggingface", "dataset": hf_dataset, "config": hf_config, "revision": revision,
                  "shards": sorted(shards), "shard_sha256": {k: v.lower() for k, v in hf_shard_checksums.items()}}
        records = _records_parquet(verified)
    heldout = _heldout_keys(exclude_validation_manifest) if exclude_validation_manifest else None
    excluded = 0
    seen: dict[str, str] = {}
    candidates = []  # (rank, id, text, source_offset, content_hash)
    scanned = 0
    for rec, offset in records:
        scanned += 1
        text = rec.get("text")
        if not isinstance(text, str):
            raise ValueError("every record requires string text")
        content = _digest(text)
        stable = rec.get("id", rec.get("doc_id"))
        doc_id = content if stable is None else str(stable)
        if doc_id in seen:
            if seen[doc_id] != content:
                raise ValueError(f"conflicting content for duplicate document ID: {doc_id}")
            continue
        seen[doc_id] = content
        if heldout is not None:
            processed = _digest(text.replace("\r\n", "\n").replace("\r", "\n")) if "\r" in text else content
            if ("id", doc_id) in heldout or ("raw", content) in heldout or ("processed", processed) in heldout:
                excluded += 1
                continue
        candidates.append((_digest("selection\0" + doc_id), doc_id, text, offset, content))
    candidates.sort(key=lambda c: (c[0], c[1]))
    candidates = candidates[:max_documents]
    streams = {s: (out / f"{s}.tokens.bin").open("wb") for s in SPLIT_ORDER}
    offsets = dict.fromkeys(SPLIT_ORDER, 0)
    total = count = 0
    try:
        with (out / "documents.jsonl").open("w") as meta:
            from .data_preparation import ordered_tokenization
            rows = ((doc_id, text, rank, offset, content) for rank, doc_id, text, offset, content in candidates)
            for doc_id, processed_sha, encoded, rank, offset, content in ordered_tokenization(
                    rows, tokenizer=tokenizer, workers=workers, batch_bytes=tokenization_batch_bytes):
                remaining = max_tokens - total
                eos_included = len(encoded) + 1 <= remaining
                toks = encoded[:remaining].astype(TOKEN_DTYPE)
                n = len(toks) + int(eos_included)
                split_rank = int(_digest(doc_id), 16)
                cum = 0.0
                for split, frac in fractions.items():
                    cum += frac
                    if split_rank < int(cum * 2 ** 256):
                        break
                start = offsets[split]
                toks.tofile(streams[split])
                if eos_included:
                    streams[split].write(np.asarray([EOS], dtype=TOKEN_DTYPE).tobytes())
                offsets[split] += n
                doc = {"id": doc_id, "numeric_id": count, "split": split, "selection_sha256": rank,
                       "content_sha256": content, "processed_sha256": processed_sha,
                       "source_offset": offset, "token_start": start, "token_end": offsets[split],
                       "source_token_start": 0, "source_token_end": n, "processed_token_start": 0,
                       "processed_token_end": min(n, len(encoded)),
                       "synthetic_eos_token_offset": len(encoded) if eos_included else None,
                       "truncated": not eos_included}
                meta.write(json.dumps(doc, sort_keys=True) + "\n")
                count += 1
                total += n
                if total >= max_tokens:
                    break
    finally:
        for s in streams.values():
            s.close()
    artifacts = {p.name: _sha(p) for p in sorted(out.iterdir()) if p.is_file()}
    manifest = {"format_version": 1, "source": source, "tokenizer": tok_meta, "split_fractions": fractions,
                "split_order": list(SPLIT_ORDER), "tokens": offsets, "documents": count, "scan_records": scanned,
                "scan_unique_documents": len(seen), "max_tokens": max_tokens, "max_documents": max_documents,
                "preprocessing": "CRLF/CR to LF; otherwise unchanged",
                "deduplication": "identical stable-ID/content duplicates collapse; conflicting contents rejected",
                "membership": "SHA256(UTF8(stable document ID)), fixed fraction intervals",
                "hash_domains": {"selection": "UTF8(selection + NUL + stable document ID)",
                                 "split": "UTF8(stable document ID)"},
                "bounded_selection": "smallest domain-separated selection SHA256 ranks across entire declared "
                                     "source; canonical rank order then token cap",
                # The two descriptive strings below are the reference's wording, byte for byte: the
                # manifest's sha256 is the dataset identity that checkpoints and resumes compare, so
                # the same source must give the same manifest in both frameworks.
                "token_offset_semantics": ("source_token_* are legacy processed document stream offsets including "
                                           "synthetic EOS; processed_token_* exclude EOS; no original "
                                           "character/byte alignment"),
                "preparation_cost": ("full declared source scan and HF raw-shard download/hash; output "
                                     "token/document bounds do not bound scan cost"),
                "boundary_loss_policy": "ignore cross-document transitions and padding", "artifacts": artifacts}
    if heldout is not None:
        manifest["heldout_exclusion"] = {"excluded_unique_documents": excluded,
                                         "rule": "exclude validation IDs and raw/processed content hashes"}
    text = json.dumps(manifest, sort_keys=True, indent=2) + "\n"
    (out / "manifest.sha256").write_text(_digest(text) + "\n")
    for p in out.iterdir():
        with p.open("rb") as fh:
            os.fsync(fh.fileno())
    from .sampler_index import ensure_sampler_index
    ensure_sampler_index(out, manifest)
    tmp = out / ".manifest.json.tmp"
    with tmp.open("w") as fh:
        fh.write(text)
        fh.flush()
        os.fsync(fh.fileno())
    os.replace(tmp, out / "manifest.json")
    return out / "manifest.json"


# ------------------------------------------------------------------------------------------ sampler
class _RowArithmetic:
    """Where the rows of a packed stream begin and end, computed without materialising them.

    Rows hold ``width = context + 1`` tokens.  Documents are laid down in epoch order; a document
    that reaches the end of a row with tokens left continues in the next row, whose first token
    repeats the row's last one.  A document of ``length`` tokens entering a row that already holds
    ``fill`` tokens either stays open (``length < width - fill``) or closes that row after
    ``width - fill`` of its tokens and then one continuation row per further ``context`` tokens;
    a remainder ``r > 0`` leaves an open row holding ``r + 1`` tokens (the repeated one included),
    a zero remainder leaves no open row."""

    def __init__(self, context: int, length_of):
        self.context, self.width, self.length_of = context, context + 1, length_of

    def after(self, length: int, rows: int, fill: int) -> tuple[int, int]:
        """(completed rows, fill of the open row) after appending ``length`` tokens of one document."""
        room = self.width - fill
        if length < room:
            return rows, fill + length
        continuation, left = divmod(length - room, self.context)
        return rows + 1 + continuation, (left + 1 if left else 0)

    def after_documents(self, order, count=None) -> tuple[int, int]:
        rows = fill = 0
        for i in (order if count is None else order[:count]):
            rows, fill = self.after(self.length_of(int(i)), rows, fill)
        return rows, fill

    def rows_in_epoch(self, order) -> int:
        rows, fill = self.after_documents(order)
        return rows + bool(fill)

    def row_start(self, order, row: int) -> tuple[int, int]:
        """(document position, token offset) at which row ``row`` begins; (len(order), 0) once the
        epoch's rows are used up."""
        rows = fill = 0
        for d in range(len(order)):
            if rows == row and fill == 0:
                return d, 0
            length = self.length_of(int(order[d]))
            done, next_fill = self.after(length, rows, fill)
            if rows < row <= done:  # an earlier row closes inside this document
                consumed = (self.width - fill) + (row - rows - 1) * self.context
                return (d, consumed - 1) if consumed < length else (d + 1, 0)
            rows, fill = done, next_fill
        if row == rows + bool(fill):
            return len(order), 0
        raise ValueError("invalid canonical row seek")

    def row_holding(self, order, document: int, token: int) -> int:
        """Index of the row in which token ``token`` of the document at position ``document`` first
        appears (it may close that row and repeat at the start of the next)."""
        rows, fill = self.after_documents(order, document)
        return self.after(token + 1, rows, fill)[0]


class PackedSampler:
    """Deterministic epoch permutations, row packing and a resumable next-batch order.

    The stream position is (epoch, row cursor, document position, token offset); the last two are
    where the next row begins and are always ``_RowArithmetic.row_start`` of the row cursor, which
    ``load_state_dict`` checks.  A context fork restarts the stream at the new context's row holding
    the old stream's next token; targets at or before that watermark are masked in the first row."""

    _STATE_KEYS = ("packing_version", "manifest_hash", "split", "batch_size", "context", "seed", "epoch", "cursor",
                   "document_cursor", "token_cursor")
    _IDENTITY_KEYS = ("packing_version", "manifest_hash", "split", "batch_size", "context", "seed")

    def __init__(self, manifest, split="train", batch_size=1, context=512, seed=0):
        self.path = _manifest_path(manifest)
        self.manifest_hash = manifest_hash(self.path)
        self.manifest = json.loads(self.path.read_text())
        self._check_dataset(split, batch_size, context)
        self.split, self.batch_size, self.context, self.seed = split, batch_size, context, seed
        from .sampler_index import load_sampler_index
        root = self.path.parent
        self.docs = load_sampler_index(root, self.manifest, split)
        if len(self.docs) == 0:
            raise ValueError(f"empty split: {split}")
        self.tokens = read_split_tokens(root, split)
        self.packing_version = PACKING_VERSION
        self._orders: dict[int, np.ndarray] = {}
        self.epoch = self.cursor = 0
        self._start_epoch()
        self._batch_mappings = []

    def _check_dataset(self, split, batch_size, context):
        root, manifest = self.path.parent, self.manifest
        for name, expected in manifest["artifacts"].items():
            if Path(name).name != name or _sha(root / name) != expected:
                raise ValueError(f"artifact checksum mismatch: {name}")
        if split not in manifest["tokens"] or batch_size <= 0 or context <= 0:
            raise ValueError("invalid split or batch shape")
        if not {"documents.jsonl", *(f"{s}.tokens.bin" for s in SPLIT_ORDER)} <= manifest["artifacts"].keys():
            raise ValueError("dataset manifest lacks required metadata/token artifacts")
        if manifest.get("format_version") != 1:
            raise ValueError("unsupported dataset format")
        counts = manifest["tokens"]
        if set(counts) != set(SPLIT_ORDER) or any(type(n) is not int or n < 0 for n in counts.values()):
            raise ValueError("invalid dataset token counts")
        for name, n in counts.items():
            if (root / f"{name}.tokens.bin").stat().st_size != n * np.dtype(TOKEN_DTYPE).itemsize:
                raise ValueError(f"token payload size mismatch: {name}")

    # ---------------------------------------------------------------- epochs and rows
    @property
    def _rows(self) -> _RowArithmetic:
        return _RowArithmetic(self.context, self.docs.length)

    def _order_of(self, epoch: int) -> np.ndarray:
        """The epoch's document order: ``random.Random(f"{seed}:{epoch}")`` shuffles positions."""
        order = self._orders.get(epoch)
        if order is None:
            order = np.arange(len(self.docs), dtype=np.int64)
            random.Random(f"{self.seed}:{epoch}").shuffle(order)
            order.flags.writeable = False
            self._orders = {epoch: order}  # one epoch is live at a time
        return order

    def _start_epoch(self):
        self._context_transition = None
        self.order = self._order_of(self.epoch)
        self.epoch_row_count = self._rows.rows_in_epoch(self.order)
        self.document_cursor = self.token_cursor = 0

    def _take_row(self) -> list[tuple[int, int, int]]:
        """The next row's pieces (document index, first token in the split file, token count);
        moves the document/token position to the next row's start."""
        pieces, fill, width = [], 0, self.context + 1
        while self.document_cursor < len(self.order) and fill < width:
            doc = int(self.order[self.document_cursor])
            length = self.docs.length(doc)
            count = min(width - fill, length - self.token_cursor)
            pieces.append((doc, self.docs.start(doc) + self.token_cursor, count))
            fill += count
            self.token_cursor += count
            if self.token_cursor == length:
                self.document_cursor, self.token_cursor = self.document_cursor + 1, 0
            elif fill == width:
                self.token_cursor -= 1  # repeated as the next row's first token
        return pieces

    def _advance(self):
        """Take one row (rolling over to the next epoch first if needed); returns (pieces, pending
        context transition, document position where the row began)."""
        if self.cursor >= self.epoch_row_count:
            self.epoch, self.cursor = self.epoch + 1, 0
            self._start_epoch()
        transition, first_document = self._context_transition, self.document_cursor
        pieces = self._take_row()
        self._context_transition = None
        self.cursor += 1
        return pieces, transition, first_document

    # ---------------------------------------------------------------- batches
    def _row_contents(self, pieces):
        """(token list, document id list, per-piece mapping records) of one row."""
        tokens, doc_ids, mappings = [], [], []
        for doc, start, count in pieces:
            rec = self.docs[doc]
            packed = len(tokens)
            offset = start - rec["token_start"]
            mappings.append({"document_id": rec["id"], "numeric_id": rec["numeric_id"],
                             "content_sha256": rec["content_sha256"], "processed_sha256": rec["processed_sha256"],
                             "source_offset": rec["source_offset"],
                             "synthetic_eos_token_offset": rec["synthetic_eos_token_offset"],
                             "processed_document_token_count": rec["processed_token_end"],
                             "packed_token_start": packed, "packed_token_end": packed + count,
                             "source_token_start": offset, "source_token_end": offset + count})
            tokens.extend(self.tokens[start:start + count].tolist())
            doc_ids.extend([self.docs.numeric_id(doc)] * count)
        return tokens, doc_ids, mappings

    def next_batch(self):
        """(inputs, document ids, targets), each [batch_size, context]; padding uses EOS inputs,
        distinct negative document ids and -100 targets; targets never cross documents."""
        shape = (self.batch_size, self.context)
        idx = torch.full(shape, EOS, dtype=torch.long)
        ids = torch.full(shape, -1, dtype=torch.long)
        targets = torch.full(shape, -100, dtype=torch.long)
        self._batch_mappings = []
        for b in range(self.batch_size):
            pieces, transition, first_document = self._advance()
            tokens, doc_ids, mappings = self._row_contents(pieces)
            n = min(self.context, len(tokens))
            self._batch_mappings.append({"epoch": self.epoch, "row_cursor": self.cursor - 1, "input_length": n,
                                         "ranges": mappings})
            row_tokens = torch.tensor(tokens, dtype=torch.long)
            row_docs = torch.tensor(doc_ids, dtype=torch.long)
            idx[b, :n], ids[b, :n] = row_tokens[:n], row_docs[:n]
            scored = min(self.context, len(tokens) - 1)
            if scored > 0:
                same = row_docs[:scored] == row_docs[1:scored + 1]
                targets[b, :scored] = torch.where(same, row_tokens[1:scored + 1], -100)
            if transition is not None:
                self._mask_replayed(b, n, targets, mappings, first_document, transition)
            if n < self.context:
                ids[b, n:] = -torch.arange(1, self.context - n + 1)
        return idx, ids, targets

    def _mask_replayed(self, b, n, targets, mappings, first_document, transition):
        """First row after a context fork: mask targets at or before the old stream's watermark and
        count the replayed inputs and masked targets."""
        *_, mark_document, mark_token = self._fork_position(transition["source_state"])

        def seen(position, offset):
            return position < mark_document or (position == mark_document and offset <= mark_token)
        replayed = masked = 0
        for k, m in enumerate(mappings):
            position, first = first_document + k, m["packed_token_start"]
            base = m["source_token_start"] - first
            replayed += sum(seen(position, base + col) for col in range(first, min(n, m["packed_token_end"])))
            for col in range(first, min(self.context, m["packed_token_end"] - 1)):
                if seen(position, base + col + 1):
                    masked += int(targets[b, col] != -100)
                    targets[b, col] = -100
        self._batch_mappings[-1]["context_fork_exposure"] = {"prefix_tokens_at_or_before_watermark": replayed,
                                                             "masked_prediction_targets": masked}

    def batch_mappings(self):
        return copy.deepcopy(self._batch_mappings)

    def batch_context_exposure(self):
        keys = ("prefix_tokens_at_or_before_watermark", "masked_prediction_targets")
        return {k: sum(r.get("context_fork_exposure", {}).get(k, 0) for r in self._batch_mappings) for k in keys}

    __next__ = next_batch

    def __iter__(self):
        return self

    # ---------------------------------------------------------------- context forks
    def _fork_position(self, source):
        """(epoch, row cursor, row start document, row start token, watermark document, watermark
        token) of this sampler's context resuming after ``source``'s consumed targets."""
        epoch, mark_document, mark_token = source["epoch"], source["document_cursor"], source["token_cursor"]
        order = self._order_of(epoch)
        if mark_document == len(order):  # the source had finished its epoch
            epoch, mark_document, mark_token = epoch + 1, 0, 0
            order = self._order_of(epoch)
        rows = self._rows
        cursor = rows.row_holding(order, mark_document, mark_token)
        start_document, start_token = rows.row_start(order, cursor)
        return epoch, cursor, start_document, start_token, mark_document, mark_token

    def fork_context(self, context):
        """A stream at a larger (or equal) context that continues after the consumed targets:
        earlier inputs may replay as prefix, but their targets are masked once."""
        if type(context) is not int or context <= 0:
            raise ValueError("context must be a positive integer")
        current = PackedSampler.state_dict(self)
        same = copy.copy(self)
        PackedSampler.load_state_dict(same, current)
        if context == self.context:
            return same
        pending = current.get("context_transition")
        source = copy.deepcopy(pending["source_state"] if pending else current)
        fork = copy.copy(self)
        fork.context = context
        epoch, cursor, document, token, _, _ = fork._fork_position(source)
        PackedSampler.load_state_dict(fork, {
            **source, "context": context, "epoch": epoch, "cursor": cursor, "document_cursor": document,
            "token_cursor": token,
            "context_transition": {"version": 1, "source_context": source["context"], "source_state": source}})
        return fork

    # ---------------------------------------------------------------- state
    def state_dict(self):
        state = {k: getattr(self, k) for k in self._STATE_KEYS}
        if self._context_transition is not None:
            state["context_transition"] = copy.deepcopy(self._context_transition)
        return state

    def _check_transition(self, transition, position):
        if (not isinstance(transition, dict) or set(transition) != {"version", "source_context", "source_state"}
                or transition["version"] != 1):
            raise ValueError("invalid context transition schema")
        source, source_context = transition["source_state"], transition["source_context"]
        if (type(source_context) is not int or source_context <= 0 or not isinstance(source, dict)
                or source.get("context") != source_context or set(source) != set(self._STATE_KEYS)):
            raise ValueError("invalid context transition source")
        at_source = copy.copy(self)
        at_source.context, at_source._context_transition = source_context, None
        PackedSampler.load_state_dict(at_source, source)
        if position != self._fork_position(source)[:4]:
            raise ValueError("context transition cursor mismatch")

    def load_state_dict(self, state):
        for k in self._IDENTITY_KEYS:
            if state.get(k) != getattr(self, k):
                raise ValueError(f"sampler state mismatch: {k}")
        position = tuple(state[k] for k in ("epoch", "cursor", "document_cursor", "token_cursor"))
        if any(type(v) is not int or v < 0 for v in position):
            raise ValueError("invalid sampler cursor")
        epoch, cursor, document, token = position
        order = self._order_of(epoch)
        rows = self._rows
        total = rows.rows_in_epoch(order)
        if cursor > total or document > len(order):
            raise ValueError("invalid sampler cursor")
        if document < len(order) and token >= self.docs.length(int(order[document])):
            raise ValueError("invalid document token cursor")
        if rows.row_start(order, cursor) != (document, token):
            raise ValueError("inconsistent row/document/token cursors")
        transition = copy.deepcopy(state.get("context_transition"))
        if transition is not None:
            self._check_transition(transition, position)
        self.epoch, self.order, self.epoch_row_count = epoch, self._order_of(epoch), total
        self.cursor, self.document_cursor, self.token_cursor = cursor, document, token
        self._context_transition = transition
        self._batch_mappings = []


class RankPackedSampler(PackedSampler):
    """This rank's contiguous slice of one global packed-row stream: each call consumes
    ``world_size * batch_size`` rows and materialises only this rank's rows."""

    def __init__(self, manifest, *, rank, world_size, split="train", batch_size=1, context=512, seed=0):
        if type(world_size) is not int or world_size < 1 or type(rank) is not int or not 0 <= rank < world_size:
            raise ValueError("invalid sampler rank/world_size")
        if type(batch_size) is not int or batch_size < 1:
            raise ValueError("batch_size must be a positive integer")
        self.rank, self.world_size = rank, world_size
        super().__init__(manifest, split=split, batch_size=batch_size, context=context, seed=seed)

    def _skip(self, rows: int):
        for _ in range(rows):
            self._advance()

    def next_batch(self):
        self._skip(self.rank * self.batch_size)
        batch = super().next_batch()
        self._skip((self.world_size - self.rank - 1) * self.batch_size)
        return batch

    __next__ = next_batch

    def state_dict(self):
        return {"rank_packing_version": 1, "rank": self.rank, "world_size": self.world_size,
                "stream": super().state_dict()}

    def load_state_dict(self, state):
        for key, expected in (("rank_packing_version", 1), ("rank", self.rank), ("world_size", self.world_size)):
            if type(state.get(key)) is not int or state[key] != expected:
                raise ValueError(f"rank sampler state mismatch: {key}")
        super().load_state_dict(state["stream"])


def batch_hash(batch) -> str:
    h = hashlib.sha256()
    values = batch.values() if isinstance(batch, dict) else batch
    for value in values:
        value = value.detach().cpu().contiguous()
        h.update(str((tuple(value.shape), str(value.dtype))).encode())
        h.update(value.numpy().tobytes())
    return h.hexdigest()


def audit_validation_overlap(training_manifest, validation_manifest, document_ids=None) -> dict:
    """Exact whole-document (raw / processed sha256) overlap of validation documents with the
    train, calibration and test splits, from metadata only."""
    fields = ("content_sha256", "processed_sha256")
    compared = ("train", "calibration", "test")
    limit = 10

    def meta(path):
        path = _manifest_path(path)
        digest = manifest_hash(path)
        expected = json.loads(path.read_text()).get("artifacts", {}).get("documents.jsonl")
        docs = path.with_name("documents.jsonl")
        if not isinstance(expected, str) or _sha(docs) != expected:
            raise ValueError("documents.jsonl artifact checksum mismatch")
        rows = [json.loads(line) for line in docs.read_text().splitlines() if line.strip()]
        return digest, rows

    th, train_rows = meta(training_manifest)
    vh, val_rows = meta(validation_manifest)
    requested = None if document_ids is None else ({document_ids} if isinstance(document_ids, str)
                                                   else {str(x) for x in document_ids})
    index = {s: {f: {} for f in fields} for s in compared}
    for d in train_rows:
        if d["split"] in index:
            for f in fields:
                index[d["split"]][f].setdefault(d[f].lower(), d["id"])
    counts = dict.fromkeys(compared, 0)
    samples = {s: [] for s in compared}
    selected, first = set(), {f: {} for f in fields}
    dup_ids, dup_hashes, dup_samples = set(), {f: set() for f in fields}, []
    for d in val_rows:
        if d["split"] != "val" or (requested is not None and d["id"] not in requested):
            continue
        selected.add(d["id"])
        for s in compared:
            hit = False
            for f in fields:
                other = index[s][f].get(d[f].lower())
                if other is not None:
                    hit = True
                    if len(samples[s]) < limit:
                        samples[s].append({"validation_document_id": d["id"], "other_document_id": other,
                                           "hash_kind": f, "sha256": d[f].lower()})
            counts[s] += int(hit)
        for f in fields:
            prev = first[f].setdefault(d[f].lower(), d["id"])
            if prev != d["id"]:
                dup_ids.update((prev, d["id"]))
                dup_hashes[f].add(d[f].lower())
                if len(dup_samples) < limit:
                    dup_samples.append({"validation_document_id": d["id"], "other_document_id": prev,
                                        "hash_kind": f, "sha256": d[f].lower()})
    if requested is not None and requested - selected:
        raise ValueError(f"unknown requested validation document IDs: {sorted(requested - selected)[:limit]}")
    return {"training_manifest_hash": th, "validation_manifest_hash": vh,
            "selected_validation_documents": len(selected),
            "selected_validation_ids_sha256": hashlib.sha256(json.dumps(sorted(selected), separators=(",", ":"))
                                                             .encode()).hexdigest(),
            "overlap_counts": counts, "overlap_samples": samples,
            "duplicate_validation": {"documents_with_duplicate_content": len(dup_ids),
                                     "hash_group_counts": {f: len(v) for f, v in dup_hashes.items()},
                                     "samples": dup_samples},
            "has_overlap": bool(any(counts.values()) or dup_ids),
            "scope": "exact whole-document original/processed SHA256 equality only", "sample_limit": limit}


def synthetic_batches(steps, rows, context, vocab, seed=0):
    """Uniform random token rows (the benchmark's data): yields (idx, doc_ids, targets) on the CPU."""
    g = torch.Generator().manual_seed(seed)
    for _ in range(steps):
        toks = torch.randint(0, vocab, (rows, context + 1), generator=g)
        yield toks[:, :-1].contiguous(), torch.zeros(rows, context, dtype=torch.long), toks[:, 1:].contiguous()
