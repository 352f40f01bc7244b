"""Sampler index (derived, verified, rebuilt when stale) and the synthetic mechanism tasks (exact labels,
held-out compositions, checksums) on CPU."""
import json
from pathlib import Path

import pytest

from helpers import FixtureTokenizer
from tensor_train_ing_b200.data import prepare_data
from tensor_train_ing_b200.sampler_index import INDEX_DIR, RECORD, index_digest, load_sampler_index
from tensor_train_ing_b200.tasks import load_mechanism_tasks, prepare_mechanism_tasks


@pytest.fixture
def dataset(tmp_path):
    source = tmp_path / "source.jsonl"
    texts = ["doc number %d %s" % (i, "x" * i) for i in range(12)]
    source.write_text("".join(json.dumps({"id": str(i), "text": t}) + "\n" for i, t in enumerate(texts)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=source, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .75, "val": .25, "test": 0., "calibration": 0.})
    return Path(manifest).parent, json.loads(Path(manifest).read_text())


def test_index_rows_match_document_metadata(dataset):
    root, manifest = dataset
    docs = [json.loads(l) for l in (root / "documents.jsonl").read_text().splitlines()]
    for split in ("train", "val"):
        idx = load_sampler_index(root, manifest, split)
        want = [d for d in docs if d["split"] == split]
        assert len(idx) == len(want)
        for i, d in enumerate(want):
            assert idx.start(i) == d["token_start"] and idx.length(i) == d["token_end"] - d["token_start"]
            assert idx.numeric_id(i) == d["numeric_id"]
            assert idx[i]["id"] == d["id"]  # the full metadata line, read by offset
    assert (root / INDEX_DIR / "train.index.bin").stat().st_size == len(load_sampler_index(root, manifest, "train")) \
        * RECORD.itemsize


def test_stale_or_corrupt_index_is_rebuilt(dataset):
    root, manifest = dataset
    load_sampler_index(root, manifest, "train")
    good = index_digest(root)
    (root / INDEX_DIR / "train.index.bin").write_bytes(b"\0" * 7)  # truncated / corrupt
    idx = load_sampler_index(root, manifest, "train")
    assert index_digest(root) == good and len(idx) > 0
    header = root / INDEX_DIR / "index.json"
    meta = json.loads(header.read_text())
    meta["identity"]["documents_sha256"] = "0" * 64  # built for other metadata
    header.write_text(json.dumps(meta))
    load_sampler_index(root, manifest, "train")
    assert json.loads(header.read_text())["identity"]["documents_sha256"] == manifest["artifacts"]["documents.jsonl"]
    assert json.loads(header.read_text())["identity"]["manifest_sha256"] == \
        (root / "manifest.sha256").read_text().strip()
    with pytest.raises(ValueError):
        load_sampler_index(root, manifest, "holdout")


def test_index_is_a_bounded_sequence(dataset):
    """Iteration stops at the end of the split, negative positions count from the end and positions
    outside the split raise IndexError (the contract ``Sequence`` iteration relies on)."""
    root, manifest = dataset
    idx = load_sampler_index(root, manifest, "train")
    ids = [d["id"] for d in idx]
    assert len(ids) == len(idx) > 1
    assert idx[-1]["id"] == ids[-1] and idx.start(-1) == idx.start(len(idx) - 1)
    for bad in (len(idx), -len(idx) - 1):
        with pytest.raises(IndexError):
            idx[bad]
        with pytest.raises(IndexError):
            idx.length(bad)
    assert [d["id"] for d in idx[1:3]] == ids[1:3]


def test_page_release_keeps_the_sampler_stream(dataset):
    """Releasing the mapping's resident pages (periodically or by hand) changes no value the
    sampler reads: two samplers, one releasing after every row read, give the same batches."""
    from tensor_train_ing_b200.data import PackedSampler
    root, manifest = dataset
    plain = PackedSampler(root / "manifest.json", batch_size=2, context=6, seed=4)
    released = PackedSampler(root / "manifest.json", batch_size=2, context=6, seed=4)
    released.docs.RELEASE_EVERY = 1
    for _ in range(8):
        a, b = plain.next_batch(), released.next_batch()
        for x, y in zip(a, b):
            assert (x == y).all()
    assert released.docs.releases > 0 and plain.docs.releases == 0
    assert released.docs.release_pages() is True and released.docs.reads == 0


def test_page_release_counts_reads_and_is_safe_without_madvise(dataset, monkeypatch):
    import mmap
    root, manifest = dataset
    idx = load_sampler_index(root, manifest, "train")
    idx.RELEASE_EVERY = 5
    calls = []
    real = idx.release_pages
    monkeypatch.setattr(idx, "release_pages", lambda: calls.append(idx.reads) or real())
    for i in range(12):
        idx.length(i % len(idx))
    assert calls == [5, 5]  # two releases after five reads each, the count reset by each
    monkeypatch.undo()
    before = [idx.start(i) for i in range(len(idx))]
    monkeypatch.delattr(mmap, "MADV_DONTNEED")
    assert idx.release_pages() is False  # no such advice here: nothing released, nothing changed
    assert [idx.start(i) for i in range(len(idx))] == before


def test_concurrent_builds_publish_one_valid_index(dataset):
    """Ranks that find no index at once serialise on the dataset's lock: one builds, the others
    find it valid, and every one reads the same rows."""
    import threading
    root, manifest = dataset
    loaded, errors = [], []

    def load():
        try:
            loaded.append([idx.start(i) for idx in [load_sampler_index(root, manifest, "train")]
                           for i in range(len(idx))])
        except Exception as exc:  # pragma: no cover - reported below
            errors.append(exc)
    threads = [threading.Thread(target=load) for _ in range(6)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors and len(loaded) == 6 and all(x == loaded[0] for x in loaded)
    leftovers = [p.name for p in (root / INDEX_DIR).iterdir() if p.name.startswith(".")]
    assert leftovers == []  # no temporary file of an interrupted publication


def test_the_index_is_derived_data_outside_the_manifest(dataset):
    """Building or rebuilding the index leaves the dataset's manifest and its digest untouched and is
    not one of its artifacts; a dataset whose metadata no longer matches its manifest is refused by
    the sampler even when a valid-looking index exists."""
    from tensor_train_ing_b200.data import PackedSampler
    root, manifest = dataset
    before = {n: (root / n).read_bytes() for n in ("manifest.json", "manifest.sha256")}
    load_sampler_index(root, manifest, "train", rebuild=True)
    assert {n: (root / n).read_bytes() for n in before} == before
    assert not any(name.startswith(INDEX_DIR) for name in manifest["artifacts"])
    PackedSampler(root / "manifest.json", batch_size=1, context=8)  # builds or reuses the index
    docs = root / "documents.jsonl"
    docs.write_text(docs.read_text().replace('"split"', '"split" ', 1))  # same records, other bytes
    with pytest.raises(ValueError, match="checksum"):
        PackedSampler(root / "manifest.json", batch_size=1, context=8)


def test_mechanism_tasks_exact_labels_and_held_out_compositions(tmp_path):
    manifest = prepare_mechanism_tasks(tmp_path / "mech", seed=3, train_examples=8, validation_examples=8)
    meta, val = load_mechanism_tasks(manifest, "val")
    _, train = load_mechanism_tasks(manifest, "train")
    assert len(val) == 16 and len(train) == 16  # counts are per task (two tasks)
    for r in val:
        if r["task"] == "boolean_hierarchy":
            b, ops = r["bits"], r["operators"]
            f = lambda op, x, y: x ^ y if op == "xor" else x & y  # noqa: E731
            assert r["answer"] == f" {f(ops[2], f(ops[0], b[0], b[1]), f(ops[1], b[2], b[3]))}"
        else:
            assert r["answer"] == f" {dict(r['key_values'])[r['query']]}"
        assert r["text"] == r["prompt"] + r["answer"]
    for task in ("boolean_hierarchy", "associative_retrieval"):
        tr = {r["composition_id"] for r in train if r["task"] == task}
        va = {r["composition_id"] for r in val if r["task"] == task}
        assert tr and va and not tr & va  # compositions held out
    assert sum(r["answer"] == " 1" for r in val if r["task"] == "boolean_hierarchy") == 4  # balanced labels


def test_mechanism_tasks_reject_tampering_and_bad_sizes(tmp_path):
    manifest = prepare_mechanism_tasks(tmp_path / "mech", seed=0, train_examples=8, validation_examples=8)
    val = Path(manifest).with_name("val.jsonl")
    rows = val.read_text().splitlines()
    r = json.loads(rows[0])
    r["answer"] = " 9"
    val.write_text("\n".join([json.dumps(r, sort_keys=True)] + rows[1:]) + "\n")
    with pytest.raises(ValueError):
        load_mechanism_tasks(manifest, "val")
    with pytest.raises(ValueError):
        prepare_mechanism_tasks(tmp_path / "odd", train_examples=9)
    with pytest.raises(ValueError):
        prepare_mechanism_tasks(tmp_path / "big", validation_examples=44)


def test_mechanism_tasks_are_a_function_of_their_seed(tmp_path):
    a = prepare_mechanism_tasks(tmp_path / "a", seed=5, train_examples=8, validation_examples=8)
    b = prepare_mechanism_tasks(tmp_path / "b", seed=5, train_examples=8, validation_examples=8)
    c = prepare_mechanism_tasks(tmp_path / "c", seed=6, train_examples=8, validation_examples=8)
    for name in ("train.jsonl", "val.jsonl"):
        assert Path(a).with_name(name).read_bytes() == Path(b).with_name(name).read_bytes()
        assert Path(a).with_name(name).read_bytes() != Path(c).with_name(name).read_bytes()


def test_mechanism_training_audit_finds_leaked_validation_examples(tmp_path):
    """A corpus prepared from the benchmark's own train.jsonl is verified; one that also contains a
    validation example reports that composition as overlapping."""
    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.tasks import audit_mechanism_training
    manifest = prepare_mechanism_tasks(tmp_path / "mech", seed=1, train_examples=8, validation_examples=8)
    train_src = Path(manifest).with_name("train.jsonl")
    splits = {"train": 1.0, "val": 0.0, "test": 0.0, "calibration": 0.0}
    clean = prepare_data(tmp_path / "clean", source_jsonl=train_src, revision="offline-v1",
                         tokenizer=FixtureTokenizer(), split_fractions=splits)
    report = audit_mechanism_training(manifest, clean)
    assert report["verified"] and report["status"] == "verified" and not report["has_validation_overlap"]
    assert report["coverage"]["fraction"] == 1.0
    _, val = load_mechanism_tasks(manifest, "val")
    leaked = tmp_path / "leaked.jsonl"
    leaked.write_text(train_src.read_text() + json.dumps({"id": "leak", "text": val[0]["text"]}) + "\n")
    dirty = prepare_data(tmp_path / "dirty", source_jsonl=leaked, revision="offline-v1",
                         tokenizer=FixtureTokenizer(), split_fractions=splits)
    report = audit_mechanism_training(manifest, dirty)
    assert report["status"] == "overlap" and not report["verified"]
    assert val[0]["composition_id"] in report["validation_composition_overlap"][val[0]["task"]]
