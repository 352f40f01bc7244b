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
class PackedSampler:
    """Deterministic epoch permutations, row packing and a resumable next-batch order."""

    _STATE_KEYS = ("packing_version", "manifest_hash", "split", "batch_size", "context", "seed", "epoch", "cursor",
                   "document_cursor", "token_cursor")

    def __init__(self, manifest, split="train", batch_size=1, context=512, seed=0):
        self.path = _manifest_path(manifest)
        self.manifest_hash = manifest_hash(self.path)
        self.manifest = json.loads(self.path.read_text())
        root = self.path.parent
        for name, expected in self.manifest["artifacts"].items():
            if Path(name).name != name or _sha(root / name) != expected:
                raise ValueError(f"artifact checksum mismatch: {name}")
        if split not in self.manifest["tokens"] or batch_size <= 0 or context <= 0:
            raise ValueError("invalid split or batch shape")
        required = {"documents.jsonl", *(f"{s}.tokens.bin" for s in SPLIT_ORDER)}
        if not required.issubset(self.manifest["artifacts"]):
            raise ValueError("dataset manifest lacks required metadata/token artifacts")
        if self.manifest.get("format_version") != 1:
            raise ValueError("unsupported dataset format")
        counts = self.manifest["tokens"]
        if set(counts) != set(SPLIT_ORDER) or any(type(n) is not int or n < 0 for n in counts.values()):
            raise ValueError("invalid dataset token counts")
        for name, n in counts.items():
            if (root / f"{name}.tokens.bin").stat().st_size != n * np.dtype(TOKEN_DTYPE).itemsize:
                raise ValueError(f"token payload size mismatch: {name}")
        self.split, self.batch_size, self.context, self.seed = split, batch_size, context, seed
        from .sampler_index import load_sampler_index
        self.docs = load_sampler_index(root, self.manifest, split)
        if len(self.docs) == 0:
            raise ValueError(f"empty split: {split}")
        self.tokens = read_split_tokens(root, split)
        self.packing_version = PACKING_VERSION
        self.epoch = self.cursor = 0
        self._order_epoch = None
        self._new_epoch_order()
        self._batch_mappings = []
        self._context_transition = None

    # ---------------------------------------------------------------- packing arithmetic
    def _permutation(self, epoch):
        if self._order_epoch == epoch:
            return self.order
        order = np.arange(len(self.docs), dtype=np.int64)
        random.Random(f"{self.seed}:{epoch}").shuffle(order)
        order.flags.writeable = False
        return order

    def _length(self, i):
        return self.docs.length(i)

    def _count_lengths(self, lengths, *, rows=0, fill=0):
        """Rows completed (and the fill of the open row) after packing these document lengths."""
        width = self.context + 1
        for remaining in lengths:
            capacity = width - fill
            if remaining < capacity:
                fill += remaining
                continue
            rows += 1
            remaining -= capacity
            fill = 0
            if remaining:
                remaining += 1  # the overlap token starts the next row
                complete = (remaining - 1) // self.context
                rows += complete
                fill = remaining - complete * self.context
                if complete and fill == 1:
                    fill = 0
        return rows, fill

    def _epoch_rows(self, order):
        rows, fill = self._count_lengths(self._length(i) for i in order)
        return rows + bool(fill)

    def _new_epoch_order(self):
        self._context_transition = None
        self.order = self._permutation(self.epoch)
        self._order_epoch = self.epoch
        self.epoch_row_count = self._epoch_rows(self.order)
        self.document_cursor = self.token_cursor = 0

    def _prefix_count(self, order, document_cursor):
        return self._count_lengths(self._length(i) for i in order[:document_cursor])

    def _seek_row(self, order, cursor):
        """(document, token) position at which canonical row ``cursor`` starts."""
        d = t = 0
        rows = fill = 0
        remaining_rows = cursor
        width = self.context + 1
        while remaining_rows:
            if d == len(order):
                if fill and remaining_rows == 1:
                    return d, 0
                raise ValueError("invalid canonical row seek")
            length = self._length(order[d])
            remaining = length - t
            if fill == 0 and remaining >= width:
                count = min(remaining_rows, (remaining - 1) // self.context)
                t += count * self.context
                remaining_rows -= count
                if t == length - 1:
                    d, t = d + 1, 0
                continue
            capacity = width - fill
            if remaining < capacity:
                fill += remaining
                d, t = d + 1, 0
            else:
                if remaining == capacity:
                    d, t = d + 1, 0
                else:
                    t += capacity - 1
                remaining_rows -= 1
                fill = 0
        return d, t

    def _fork_position(self, source):
        epoch, d, t = source["epoch"], source["document_cursor"], source["token_cursor"]
        order = self._permutation(epoch)
        if d == len(order):
            epoch, d, t = epoch + 1, 0, 0
            order = self._permutation(epoch)
        rows, fill = self._prefix_count(order, d)
        cursor, _ = self._count_lengths((t + 1,), rows=rows, fill=fill)
        dc, tc = self._seek_row(order, cursor)
        return epoch, cursor, dc, tc, d, t

    def fork_context(self, context):
        """New stream at a larger (or equal) context that continues after the consumed targets:
        earlier inputs may replay as prefix but their targets are masked once."""
        if type(context) is not int or context <= 0:
            raise ValueError("context must be a positive integer")
        original = PackedSampler.state_dict(self)
        check = copy.copy(self)
        PackedSampler.load_state_dict(check, original)
        if context == self.context:
            return check
        transition = original.get("context_transition")
        source = copy.deepcopy(transition["source_state"] if transition else original)
        fork = copy.copy(self)
        fork.context = context
        fork._order_epoch = None
        epoch, cursor, d, t, _, _ = fork._fork_position(source)
        target = {**source, "context": context, "epoch": epoch, "cursor": cursor, "document_cursor": d,
                  "token_cursor": t, "context_transition": {"version": 1, "source_context": source["context"],
                                                            "source_state": source}}
        PackedSampler.load_state_dict(fork, target)
        return fork

    # ---------------------------------------------------------------- batches
    def _next_row(self):
        row, fill = [], 0
        width = self.context + 1
        while self.document_cursor < len(self.order) and fill < width:
            i = int(self.order[self.document_cursor])
            length = self._length(i)
            count = min(width - fill, length - self.token_cursor)
            row.append((i, self.docs.start(i) + self.token_cursor, count))
            fill += count
            self.token_cursor += count
            if self.token_cursor == length:
                self.document_cursor += 1
                self.token_cursor = 0
            elif fill == width:
                self.token_cursor -= 1
        return row

    def next_batch(self):
        idx = torch.full((self.batch_size, self.context), EOS, dtype=torch.long)
        ids = torch.full_like(idx, -1)
        targets = torch.full_like(idx, -100)
        self._batch_mappings = []
        for b in range(self.batch_size):
            if self.cursor >= self.epoch_row_count:
                self.epoch += 1
                self.cursor = 0
                self._new_epoch_order()
            transition = self._context_transition
            row_start_document = self.document_cursor
            row = self._next_row()
            self._context_transition = None
            self.cursor += 1
            tok, docids, mappings = [], [], []
            for i, start, count in row:
                doc = self.docs[i]
                packed_start = len(tok)
                mappings.append({"document_id": doc["id"], "numeric_id": doc["numeric_id"],
                                 "content_sha256": doc["content_sha256"], "processed_sha256": doc["processed_sha256"],
                                 "source_offset": doc["source_offset"],
                                 "synthetic_eos_token_offset": doc["synthetic_eos_token_offset"],
                                 "processed_document_token_count": doc["processed_token_end"],
                                 "packed_token_start": packed_start, "packed_token_end": packed_start + count,
                                 "source_token_start": start - doc["token_start"],
                                 "source_token_end": start - doc["token_start"] + count})
                tok.extend(self.tokens[start:start + count].tolist())
                docids.extend([self.docs.numeric_id(i)] * count)
            self._batch_mappings.append({"epoch": self.epoch, "row_cursor": self.cursor - 1,
                                         "input_length": min(self.context, len(tok)), "ranges": mappings})
            n = min(self.context, len(tok))
            token_row = torch.tensor(tok, dtype=torch.long)
            doc_row = torch.tensor(docids, dtype=torch.long)
            idx[b, :n] = token_row[:n]
            ids[b, :n] = doc_row[:n]
            pairs = min(self.context, len(tok) - 1)
            if pairs > 0:
                same = doc_row[:pairs] == doc_row[1:pairs + 1]
                targets[b, :pairs] = torch.where(same, token_row[1:pairs + 1], -100)
            if transition is not None:
                self._mask_replayed(b, n, targets, mappings, row_start_document, transition)
            if n < self.context:
                ids[b, n:] = -torch.arange(1, self.context - n + 1)
        return idx, ids, targets

    def _mask_replayed(self, b, n, targets, mappings, row_start_document, transition):
        _, _, _, _, frontier_doc, frontier_tok = self._fork_position(transition["source_state"])
        exposure = {"prefix_tokens_at_or_before_watermark": 0, "masked_prediction_targets": 0}
        for k, m in enumerate(mappings):
            position = row_start_document + k
            for packed in range(m["packed_token_start"], min(n, m["packed_token_end"])):
                off = m["source_token_start"] + packed - m["packed_token_start"]
                if position < frontier_doc or (position == frontier_doc and off <= frontier_tok):
                    exposure["prefix_tokens_at_or_before_watermark"] += 1
            for packed in range(m["packed_token_start"], min(self.context, m["packed_token_end"] - 1)):
                toff = m["source_token_start"] + packed - m["packed_token_start"] + 1
                if position < frontier_doc or (position == frontier_doc and toff <= frontier_tok):
                    exposure["masked_prediction_targets"] += int(targets[b, packed] != -100)
                    targets[b, packed] = -100
        self._batch_mappings[-1]["context_fork_exposure"] = exposure

    def batch_mappings(self):
        return copy.deepcopy(self._batch_mappings)

    def batch_context_exposure(self):
        keys = ("prefix_tokens_at_or_before_watermark", "masked_prediction_targets")
        return {k: sum(r.get("context_fork_exposure", {}).get(k, 0) for r in self._batch_mappings) for k in keys}

    __next__ = next_batch

    def __iter__(self):
        return self

    # ---------------------------------------------------------------- state
    def state_dict(self):
        state = {k: getattr(self, k) for k in self._STATE_KEYS}
        if self._context_transition is not None:
            state["context_transition"] = copy.deepcopy(self._context_transition)
        return state

    def load_state_dict(self, state):
        for k in ("packing_version", "manifest_hash", "split", "batch_size", "context", "seed"):
            if state.get(k) != getattr(self, k):
                raise ValueError(f"sampler state mismatch: {k}")
        epoch, cursor = state["epoch"], state["cursor"]
        dcur, tcur = state["document_cursor"], state["token_cursor"]
        if any(type(v) is not int or v < 0 for v in (epoch, cursor, dcur, tcur)):
            raise ValueError("invalid sampler cursor")
        self_order_epoch = self._order_epoch
        self._order_epoch = None
        order = self._permutation(epoch)
        self._order_epoch = self_order_epoch
        rows_total = self._epoch_rows(order)
        if cursor > rows_total or dcur > len(order):
            raise ValueError("invalid sampler cursor")
        if dcur == len(order):
            if tcur != 0 or cursor != rows_total:
                raise ValueError("inconsistent completed epoch cursor")
        else:
            length = self._length(order[dcur])
            if tcur >= length or cursor == rows_total:
                raise ValueError("invalid document token cursor")
            rows, fill = self._prefix_count(order, dcur)
            at_start = tcur == 0 and fill == 0 and rows == cursor
            if not at_start:
                rows, fill = self._count_lengths((tcur + 1,), rows=rows, fill=fill)
                if tcur >= length - 1 or fill != 0 or rows != cursor:
                    raise ValueError("inconsistent row/document/token cursors")
        transition = copy.deepcopy(state.get("context_transition"))
        if transition is not None:
            if (not isinstance(transition, dict) or set(transition) != {"version", "source_context", "source_state"}
                    or transition["version"] != 1):
                raise ValueError("invalid context transition schema")
            source, sctx = transition["source_state"], transition["source_context"]
            if (type(sctx) is not int or sctx <= 0 or not isinstance(source, dict)
                    or source.get("context") != sctx or set(source) != set(self._STATE_KEYS)):
                raise ValueError("invalid context transition source")
            checker = copy.copy(self)
            checker.context = sctx
            checker._context_transition = None
            checker._order_epoch = None
            PackedSampler.load_state_dict(checker, source)
            probe = copy.copy(self)
            probe._order_epoch = None
            if (epoch, cursor, dcur, tcur) != probe._fork_position(source)[:4]:
                raise ValueError("context transition cursor mismatch")
        self.epoch, self.order, self.epoch_row_count = epoch, order, rows_total
        self._order_epoch = epoch
        self.cursor, self.document_cursor, self.token_cursor = cursor, dcur, tcur
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

    def _skip_rows(self, count):
        for _ in range(count):
            if self.cursor >= self.epoch_row_count:
                self.epoch += 1
                self.cursor = 0
                self._new_epoch_order()
            self._next_row()
            self._context_transition = None
            self.cursor += 1

    def next_batch(self):
        self._skip_rows(self.rank * self.batch_size)
        batch = super().next_batch()
        self._skip_rows((self.world_size - self.rank - 1) * self.batch_size)
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
