"""Dataset preparation and the packed sampler: replay, boundaries, integrity, rank slicing."""
import json

import pytest
import torch

from helpers import FixtureTokenizer
from tensor_train_ing_b200.data import (PackedSampler, RankPackedSampler, audit_validation_overlap, batch_hash,
                                        manifest_hash, prepare_data)


@pytest.fixture
def dataset(tmp_path):
    src = tmp_path / "src.jsonl"
    texts = ["short", "a somewhat longer document", "xyz", "hello world", "the quick brown fox", "q"]
    src.write_text("".join(json.dumps({"id": f"d{i}", "text": t}) + "\n" for i, t in enumerate(texts * 3)))
    # duplicates by id are rejected; give each copy its own id
    rows = [json.loads(x) for x in src.read_text().splitlines()]
    src.write_text("".join(json.dumps({"id": f"doc{i}", "text": r["text"] + str(i)}) + "\n" for i, r in enumerate(rows)))
    return prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                        split_fractions={"train": .7, "val": .1, "test": .1, "calibration": .1})


def _batches(sampler, n):
    return [sampler.next_batch() for _ in range(n)]


def test_replay_and_state_roundtrip(dataset):
    a = PackedSampler(dataset, batch_size=2, context=8, seed=3)
    first = _batches(a, 3)
    saved = a.state_dict()
    rest = _batches(a, 4)
    b = PackedSampler(dataset, batch_size=2, context=8, seed=3)
    b.load_state_dict(saved)
    for x, y in zip(rest, _batches(b, 4)):
        for u, v in zip(x, y):
            assert torch.equal(u, v)
    c = PackedSampler(dataset, batch_size=2, context=8, seed=3)
    assert batch_hash(first[0]) == batch_hash(c.next_batch())


def test_targets_never_cross_documents(dataset):
    s = PackedSampler(dataset, batch_size=4, context=16, seed=0)
    for idx, docs, targets in _batches(s, 5):
        for b in range(idx.shape[0]):
            for t in range(idx.shape[1] - 1):
                if targets[b, t] != -100:
                    assert docs[b, t] == docs[b, t + 1] >= 0
                    assert targets[b, t] == idx[b, t + 1]


def test_padding_has_unique_negative_ids(dataset):
    s = PackedSampler(dataset, batch_size=1, context=4096, seed=0)
    idx, docs, targets = s.next_batch()
    pad = docs[docs < 0]
    assert pad.numel() > 0 and pad.unique().numel() == pad.numel()
    assert (targets[docs < 0] == -100).all()


def test_checksum_and_state_rejection(dataset, tmp_path):
    s = PackedSampler(dataset, batch_size=1, context=8)
    bad = dict(s.state_dict(), seed=99)
    with pytest.raises(ValueError):
        s.load_state_dict(bad)
    root = dataset.parent if dataset.is_file() else dataset
    tokens = root / "train.tokens.bin"
    raw = bytearray(tokens.read_bytes())
    raw[0] ^= 1
    tokens.write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        PackedSampler(dataset, batch_size=1, context=8)


def test_rank_sampler_slices_the_global_stream(dataset):
    world, rows = 3, 2
    glob = PackedSampler(dataset, batch_size=world * rows, context=8, seed=5)
    ranks = [RankPackedSampler(dataset, rank=r, world_size=world, batch_size=rows, context=8, seed=5)
             for r in range(world)]
    for _ in range(3):
        g = glob.next_batch()
        parts = [rs.next_batch() for rs in ranks]
        for k in range(3):
            assert torch.equal(torch.cat([p[k] for p in parts]), g[k])


def test_manifest_hash_is_stable_and_overlap_audit_clean(dataset):
    assert manifest_hash(dataset) == manifest_hash(dataset)
    audit = audit_validation_overlap(dataset, dataset)
    assert audit["has_overlap"] is False


def test_failed_preparation_cleans_output(tmp_path):
    src = tmp_path / "src.jsonl"
    src.write_text(json.dumps({"id": "a", "text": "x"}) + "\n")
    with pytest.raises(ValueError):
        prepare_data(tmp_path / "out", source_jsonl=src, revision="main", tokenizer=FixtureTokenizer())
    assert not (tmp_path / "out").exists()


def test_parallel_tokenization_is_byte_identical(tmp_path):
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"d{i}", "text": ("word%d " % i) * (1 + i % 7)}) + "\n" for i in range(300)))
    outs = []
    for workers in (1, 3):
        m = prepare_data(tmp_path / f"data{workers}", source_jsonl=src, revision="offline-v1",
                         tokenizer=FixtureTokenizer(), workers=workers, tokenization_batch_bytes=256,
                         split_fractions={"train": .7, "val": .1, "test": .1, "calibration": .1})
        root = m.parent if m.is_file() else m
        outs.append({p.name: p.read_bytes() for p in root.iterdir() if p.is_file() and p.name != "manifest.json"})
    assert outs[0] == outs[1]


@pytest.mark.parametrize("context", [1, 2, 3, 5, 8, 13])
def test_row_arithmetic_matches_the_materialised_stream(dataset, context):
    """Row counts and row starts computed in closed form agree with the rows actually taken, and
    every token of every document appears as a fresh (non-repeated) input exactly once per epoch."""
    s = PackedSampler(dataset, batch_size=1, context=context, seed=5)
    rows = s._rows
    fresh = {}
    for row in range(s.epoch_row_count):
        assert (s.document_cursor, s.token_cursor) == rows.row_start(s.order, row) and s.cursor == row
        s.next_batch()
        for m in s.batch_mappings()[0]["ranges"]:
            first = m["source_token_start"] + (1 if fresh.get(m["document_id"], 0) > m["source_token_start"] else 0)
            for off in range(first, m["source_token_end"]):
                assert fresh.get(m["document_id"], 0) == off
                fresh[m["document_id"]] = off + 1
    assert (s.document_cursor, s.token_cursor) == (len(s.order), 0)
    assert rows.row_start(s.order, s.epoch_row_count) == (len(s.order), 0)
    assert all(fresh[s.docs[int(i)]["id"]] == s.docs.length(int(i)) for i in s.order)
