"""Dataset integrity rules and sampler coverage.

* one epoch of the packed sampler scores every within-document next-token pair of the split exactly
  once (rows overlap by one token, so no pair is lost or repeated at a row boundary), and each target
  is the document's token at that offset;
* later epochs reshuffle the document order and still cover the split;
* a validation dataset must share the training dataset's tokenizer; test-only fixtures need an
  explicit allowance; tampered manifests are refused;
* the overlap audit finds validation documents that also occur in the training splits, and a
  preparation that excludes a held-out manifest keeps those documents out.
"""
import json

import pytest

from helpers import FixtureTokenizer
from tensor_train_ing_b200.data import (PackedSampler, audit_validation_overlap, prepare_data, synthetic_batches,
                                        validate_tokenizer_compatibility)

SPLITS = {"train": .6, "val": .2, "test": .1, "calibration": .1}


def _source(path, texts):
    path.write_text("".join(json.dumps({"id": f"doc{i}", "text": t}) + "\n" for i, t in enumerate(texts)))
    return path


def _prepare(tmp_path, name, texts, **kw):
    src = _source(tmp_path / f"{name}.jsonl", texts)
    return prepare_data(tmp_path / name, source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                        split_fractions=SPLITS, **kw)


TEXTS = [f"document number {i} " + "abcdefghij"[: 1 + i % 10] * (1 + i % 4) for i in range(40)]


def _epoch_predictions(sampler):
    """(document id, predicted source offset) -> target token, over exactly one epoch of rows."""
    seen = {}
    start_epoch = sampler.epoch
    rows = 0
    while rows < sampler.epoch_row_count:
        idx, docs, tgt = sampler.next_batch()
        for b, row in enumerate(sampler.batch_mappings()):
            assert row["epoch"] == start_epoch
            for m in row["ranges"]:
                for col in range(m["packed_token_start"], min(sampler.context, m["packed_token_end"] - 1)):
                    key = (m["document_id"], m["source_token_start"] + col - m["packed_token_start"] + 1)
                    assert key not in seen, f"pair scored twice: {key}"
                    assert int(tgt[b, col]) != -100
                    seen[key] = int(tgt[b, col])
            rows += 1
            if rows == sampler.epoch_row_count:
                break
    return seen


@pytest.mark.parametrize("context", [5, 16])
def test_one_epoch_scores_every_within_document_pair_once(tmp_path, context):
    manifest = _prepare(tmp_path, "data", TEXTS)
    s = PackedSampler(manifest, batch_size=1, context=context, seed=11)
    seen = _epoch_predictions(s)
    expected = {}
    for i in range(len(s.docs)):
        rec, n, start = s.docs[i], s.docs.length(i), s.docs.start(i)
        for k in range(1, n):
            expected[(rec["id"], k)] = int(s.tokens[start + k])
    assert seen == expected


def test_epochs_reshuffle_and_each_covers_the_split(tmp_path):
    manifest = _prepare(tmp_path, "data", TEXTS)
    s = PackedSampler(manifest, batch_size=1, context=8, seed=2)
    first = list(s._order_of(0))
    second = list(s._order_of(1))
    assert sorted(first) == sorted(second) == list(range(len(s.docs)))
    assert first != second
    _epoch_predictions(s)
    assert s.epoch == 0
    s.next_batch()  # the first row of the next epoch
    assert s.epoch == 1
    again = PackedSampler(manifest, batch_size=1, context=8, seed=2)
    assert list(again._order_of(1)) == second  # the order is a function of (seed, epoch)


def test_tokenizer_compatibility_rules(tmp_path):
    a = _prepare(tmp_path, "a", TEXTS[:20])
    b = _prepare(tmp_path, "b", TEXTS[20:])
    with pytest.raises(ValueError, match="test-only"):
        validate_tokenizer_compatibility(a, b)
    report = validate_tokenizer_compatibility(a, b, allow_test_only=True)
    assert report["kind"] == "test_only_metadata_equality" and len(report["manifest_hashes"]) == 2
    # a validation set declaring another tokenizer is refused
    other = tmp_path / "c"
    other_manifest = prepare_data(other, source_jsonl=_source(tmp_path / "c.jsonl", TEXTS[:10]),
                                  revision="offline-v1", tokenizer=_RenamedTokenizer(), split_fractions=SPLITS)
    with pytest.raises(ValueError, match="tokenizer metadata mismatch"):
        validate_tokenizer_compatibility(a, other_manifest, allow_test_only=True)
    # a manifest edited after preparation no longer matches its stored digest
    path = tmp_path / "b" / "manifest.json"
    path.write_text(path.read_text().replace('"offline-v1"', '"offline-v2"'))
    with pytest.raises(ValueError, match="checksum"):
        validate_tokenizer_compatibility(a, b, allow_test_only=True)


class _RenamedTokenizer(FixtureTokenizer):
    name = "offline-renamed"


def test_overlap_audit_and_heldout_exclusion(tmp_path):
    heldout = _prepare(tmp_path, "heldout", TEXTS)
    val_texts = set()
    for line in (tmp_path / "heldout" / "documents.jsonl").read_text().splitlines():
        row = json.loads(line)
        if row["split"] == "val":
            val_texts.add(row["id"])
    assert val_texts
    # a training dataset holding the same texts under other ids (so they fall into other splits)
    # contains the held-out documents by content
    src = tmp_path / "copies.jsonl"
    src.write_text("".join(json.dumps({"id": f"copy{i}", "text": t}) + "\n" for i, t in enumerate(TEXTS)))
    same = prepare_data(tmp_path / "same", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                        split_fractions=SPLITS)
    report = audit_validation_overlap(same, heldout)
    assert report["selected_validation_documents"] == len(val_texts)
    assert report["has_overlap"] and sum(report["overlap_counts"].values()) > 0
    # excluding the held-out manifest at preparation keeps every one of them out (matched by content,
    # whatever their ids)
    clean = prepare_data(tmp_path / "clean", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                         split_fractions=SPLITS, exclude_validation_manifest=heldout)
    kept = {json.loads(line)["id"] for line in (tmp_path / "clean" / "documents.jsonl").read_text().splitlines()}
    assert kept and len(kept) == len(TEXTS) - len(val_texts)
    report = audit_validation_overlap(clean, heldout)
    assert not any(report["overlap_counts"].values())
    with pytest.raises(ValueError, match="unknown requested validation document"):
        audit_validation_overlap(clean, heldout, document_ids=["no-such-document"])


def test_synthetic_batches_are_seeded_next_token_rows():
    a = list(synthetic_batches(3, 4, 16, 100, seed=5))
    b = list(synthetic_batches(3, 4, 16, 100, seed=5))
    c = list(synthetic_batches(3, 4, 16, 100, seed=6))
    for (i1, d1, t1), (i2, d2, t2) in zip(a, b):
        assert (i1 == i2).all() and (t1 == t2).all() and (d1 == 0).all()
        assert i1.shape == t1.shape == (4, 16) and int(i1.max()) < 100 and int(i1.min()) >= 0
        assert (i1[:, 1:] == t1[:, :-1]).all()  # targets are the inputs shifted by one
    assert not all((x[0] == y[0]).all() for x, y in zip(a, c))
