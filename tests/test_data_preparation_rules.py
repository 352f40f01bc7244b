"""Dataset preparation and sampler restore rules on CPU:

* selection keeps the ``max_documents`` documents of smallest selection hash, so the prepared set
  does not depend on the order of the source; a document's split depends on its id alone, not on
  which other documents were selected;
* two source records with one id and different texts are refused, also when neither would be
  selected;
* the Hugging Face path reads local parquet shards only against explicit checksums (every shard,
  exactly) and a pinned 40-character revision; wrong bytes are refused; the result replays;
* a preparation that fails at any point, including while publishing its manifest, leaves no output;
* a sampler refuses a state from another identity or with inconsistent cursors and keeps its own
  position (its next batch is unchanged).
"""
import json
import random

import pytest

from helpers import FixtureTokenizer
from tensor_train_ing_b200 import data as data_module
from tensor_train_ing_b200.data import PackedSampler, prepare_data

SPLITS = {"train": .6, "val": .2, "test": .1, "calibration": .1}
TEXTS = {f"doc-{i}": f"text of document {i} " + "xyz"[i % 3] * (i % 7 + 1) for i in range(50)}


def _write(path, items):
    path.write_text("".join(json.dumps({"id": k, "text": t}) + "\n" for k, t in items))
    return path


def _prepare(tmp_path, name, items, **kw):
    src = _write(tmp_path / f"{name}.jsonl", items)
    return prepare_data(tmp_path / name, source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                        split_fractions=SPLITS, **kw)


def _docs(root):
    return [json.loads(x) for x in (root / "documents.jsonl").read_text().splitlines()]


def test_selection_ignores_source_order_and_splits_ignore_selection(tmp_path):
    items = list(TEXTS.items())
    shuffled = items[:]
    random.Random(3).shuffle(shuffled)
    a = _prepare(tmp_path, "a", items, max_documents=20)
    b = _prepare(tmp_path, "b", shuffled, max_documents=20)
    full = _prepare(tmp_path, "full", items)
    da, db, dfull = _docs(tmp_path / "a"), _docs(tmp_path / "b"), _docs(tmp_path / "full")
    assert [d["id"] for d in da] == [d["id"] for d in db] and len(da) == 20
    assert (tmp_path / "a" / "train.tokens.bin").read_bytes() == (tmp_path / "b" / "train.tokens.bin").read_bytes()
    split_of = {d["id"]: d["split"] for d in dfull}
    assert all(split_of[d["id"]] == d["split"] for d in da)
    assert json.loads(a.read_text())["tokens"] == json.loads(b.read_text())["tokens"]


def test_conflicting_duplicates_are_refused_even_outside_the_selection(tmp_path):
    items = list(TEXTS.items()) + [("doc-7", "a different text under an existing id")]
    with pytest.raises(ValueError):
        _prepare(tmp_path, "dup", items, max_documents=2)
    assert not (tmp_path / "dup").exists()


def _parquet(path, items):
    import pyarrow as pa
    import pyarrow.parquet as pq
    pq.write_table(pa.table({"id": [k for k, _ in items], "text": [t for _, t in items]}), path)
    return path


def test_local_parquet_shards_are_read_only_against_explicit_checksums(tmp_path):
    from tensor_train_ing_b200.hashing import file_sha256
    items = list(TEXTS.items())
    shards = {"part-0.parquet": _parquet(tmp_path / "p0.parquet", items[:25]),
              "part-1.parquet": _parquet(tmp_path / "p1.parquet", items[25:])}
    sums = {k: file_sha256(v) for k, v in shards.items()}
    kw = dict(revision="0123456789abcdef0123456789abcdef01234567", tokenizer=FixtureTokenizer(),
              split_fractions=SPLITS, hf_dataset="local/fixture", hf_data_files=list(shards),
              hf_local_shards={k: str(v) for k, v in shards.items()})
    manifest = prepare_data(tmp_path / "hf", hf_shard_checksums=sums, **kw)
    assert json.loads(manifest.read_text())["source"]["shard_sha256"] == sums
    _prepare(tmp_path, "jsonl", items)  # the same documents from a JSONL source
    assert (tmp_path / "hf" / "train.tokens.bin").read_bytes() == (tmp_path / "jsonl" / "train.tokens.bin").read_bytes()
    for bad_sums in (None, {"part-0.parquet": sums["part-0.parquet"]}, {**sums, "part-0.parquet": "0" * 64}):
        with pytest.raises(ValueError):
            prepare_data(tmp_path / "bad", hf_shard_checksums=bad_sums, **kw)
        assert not (tmp_path / "bad").exists()
    with pytest.raises(ValueError, match="40-character"):
        prepare_data(tmp_path / "bad", hf_shard_checksums=sums, **{**kw, "revision": "v1.0-short"})


def test_a_failed_manifest_publication_leaves_no_output(tmp_path, monkeypatch):
    real_replace = data_module.os.replace

    def failing(src, dst, *args, **kwargs):
        if str(dst).endswith("manifest.json"):  # the last step: publishing the manifest
            raise OSError(28, "injected: no space left while publishing")
        return real_replace(src, dst, *args, **kwargs)
    monkeypatch.setattr(data_module.os, "replace", failing)
    with pytest.raises(OSError, match="injected"):
        _prepare(tmp_path, "fail", list(TEXTS.items()))
    assert not (tmp_path / "fail").exists()


def test_a_refused_restore_keeps_the_sampler_position(tmp_path):
    manifest = _prepare(tmp_path, "data", list(TEXTS.items()))
    a = PackedSampler(manifest, batch_size=2, context=8, seed=5)
    twin = PackedSampler(manifest, batch_size=2, context=8, seed=5)
    for s in (a, twin):
        s.next_batch()
    good = a.state_dict()
    bad_states = [{**good, "seed": 6}, {**good, "context": 16}, {**good, "cursor": good["cursor"] + 1},
                  {**good, "token_cursor": 10 ** 6}, {**good, "epoch": -1}, {**good, "cursor": True}]
    for bad in bad_states:
        with pytest.raises(ValueError):
            a.load_state_dict(bad)
    assert a.state_dict() == twin.state_dict()
    for x, y in zip(a.next_batch(), twin.next_batch()):
        assert (x == y).all()
