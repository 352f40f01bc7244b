"""Exact-label synthetic mechanism tasks with whole compositions held out (reference
tnlm/tasks.py:39-386): a Boolean hierarchy ((a OP b) OP (c OP d)) and associative retrieval over a
4-key mapping.  The generator, its seeded partitions and the row identities follow the reference
so that task sets are identical for the same seed; ``audit_mechanism_training`` checks which
compositions a declared training corpus exposes."""
from __future__ import annotations

import hashlib
import itertools
import json
import os
import random
import shutil
from pathlib import Path

MECHANISM_VERSION = "exact-compositions-v1"
_MECHANISM_TASKS = ("boolean_hierarchy", "associative_retrieval")
_MECHANISM_KEYS = ("A", "B", "C", "D")


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
    path = _manifest_path(path)
    digest = _sha(path)
    if path.with_name("manifest.sha256").read_text().strip() != digest:
        raise ValueError("manifest checksum mismatch")
    return digest


def _mechanism_partitions(seed):
    boolean = list(itertools.product(("xor", "and"), repeat=3))
    mappings = list(itertools.product(range(4), repeat=4))
    random.Random(f"{MECHANISM_VERSION}:mappings:{seed}").shuffle(mappings)
    return {"boolean_hierarchy": {"train": [o for o in boolean if o.count("and") % 2 == 0],
                                  "val": [o for o in boolean if o.count("and") % 2 == 1]},
            "associative_retrieval": {"train": mappings[:192], "val": mappings[192:]}}


def _mechanism_row(task, split, composition, instance) -> dict:
    if task == "boolean_hierarchy":
        bits, ops = list(instance), list(composition)
        apply = lambda op, a, b: a ^ b if op == "xor" else a & b  # noqa: E731
        answer = apply(ops[2], apply(ops[0], *bits[:2]), apply(ops[1], *bits[2:]))
        comp_id = "boolean:" + "-".join(ops)
        prompt = (f"Compute ({bits[0]} {ops[0].upper()} {bits[1]}) {ops[2].upper()} "
                  f"({bits[2]} {ops[1].upper()} {bits[3]}). Answer:")
        structure = {"bits": bits, "operators": ops}
    else:
        mapping = list(zip(_MECHANISM_KEYS, composition))
        answer = composition[_MECHANISM_KEYS.index(instance)]
        comp_id = "retrieval:" + "".join(map(str, composition))
        prompt = "Mappings: " + ", ".join(f"{k}={v}" for k, v in mapping) + f". Query: {instance}. Answer:"
        structure = {"key_values": [list(p) for p in mapping], "query": instance}
    identity = {"task": task, "split": split, "composition_id": comp_id, **structure}
    return {"id": task + "/" + _digest(json.dumps(identity, sort_keys=True, separators=(",", ":"))), **identity,
            "prompt": prompt, "answer": f" {answer}", "text": prompt + f" {answer}"}


def _mechanism_bounds(seed, train_examples, validation_examples):
    if type(seed) is not int:
        raise ValueError("mechanism seed must be an integer")
    for name, count, maximum in (("train", train_examples, 36), ("val", validation_examples, 42)):
        if type(count) is not int or count < 8 or count > maximum or count % 2:
            raise ValueError(f"{name} examples per task must be even, >=8 and <= {maximum}; balanced unique "
                             "Boolean domain bound")


def prepare_mechanism_tasks(output_dir, seed=0, train_examples=32, validation_examples=16):
    """Write train.jsonl / val.jsonl (counts per task) plus a checksummed manifest."""
    _mechanism_bounds(seed, train_examples, validation_examples)
    parts = _mechanism_partitions(seed)
    rows = {"train": [], "val": []}
    for split, count in (("train", train_examples), ("val", validation_examples)):
        gen = random.Random(f"{MECHANISM_VERSION}:boolean:{seed}:{split}")
        selected, remaining = [], {" 0": [], " 1": []}
        for comp in parts["boolean_hierarchy"][split]:
            cands = [_mechanism_row("boolean_hierarchy", split, comp, bits) for bits in itertools.product(range(2), repeat=4)]
            for label in remaining:
                pool = [r for r in cands if r["answer"] == label]
                gen.shuffle(pool)
                selected.append(pool.pop())
                remaining[label].extend(pool)
        for label in remaining:
            gen.shuffle(remaining[label])
            selected.extend(remaining[label][:count // 2 - 4])
        gen.shuffle(selected)
        rows[split].extend(selected)
        gen = random.Random(f"{MECHANISM_VERSION}:retrieval:{seed}:{split}")
        pools = {str(v): [] for v in range(4)}
        for comp in parts["associative_retrieval"][split]:
            for key in _MECHANISM_KEYS:
                r = _mechanism_row("associative_retrieval", split, comp, key)
                pools[r["answer"].strip()].append(r)
        for pool in pools.values():
            gen.shuffle(pool)
        rows[split].extend(pools[str(i % 4)].pop() for i in range(count))
    metadata = {"format_version": 1, "generator_version": MECHANISM_VERSION, "seed": seed, "counts_are_per_task": True,
                "examples_per_task": {"train": train_examples, "val": validation_examples},
                "domain_bounds": {"boolean_assignments_total": 128, "retrieval_mapping_query_pairs_total": 1024,
                                  "balanced_boolean_max_per_split": {"train": 36, "val": 42}},
                "composition_splits": {t: {s: sorted({r["composition_id"] for r in rows[s] if r["task"] == t})
                                           for s in rows} for t in _MECHANISM_TASKS},
                # descriptive fields in the reference's wording: the manifest's sha256 identifies the
                # task set, so both frameworks must write the same bytes for the same seed and sizes
                "composition_definition": {
                    "associative_retrieval": ("full A/B/C/D to 0/1/2/3 mapping, values may repeat; seeded permutation "
                                              "of256 maps, first192 train, last64 val"),
                    "boolean_hierarchy": ("operator triple [left,right,root]; even AND count train, odd val; all four "
                                          "bits enumerated")},
                "label_definition": {
                    "associative_retrieval": "value for exact query key",
                    "boolean_hierarchy": "root(left(bit0,bit1),right(bit2,bit3)); xor is exclusive-or, and is conjunction"},
                "tokenizer": {"name": "gpt2",
                              "answer_contract": "leading-space digit 0..3; evaluator verifies exactly one token"},
                "scope": "exact-label synthetic mechanism probes with held-out compositions; no final-test or LM-quality claim"}
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=False)
    try:
        files = {}
        for split in rows:
            path = out / f"{split}.jsonl"
            with path.open("w") as fh:
                for r in rows[split]:
                    fh.write(json.dumps(r, sort_keys=True) + "\n")
                fh.flush()
                os.fsync(fh.fileno())
            files[path.name] = {"sha256": _sha(path), "bytes": path.stat().st_size}
        metadata["files"] = files
        text = json.dumps(metadata, sort_keys=True, indent=2) + "\n"
        (out / "manifest.sha256").write_text(_digest(text) + "\n")
        tmp = out / ".manifest.json.tmp"
        tmp.write_text(text)
        os.replace(tmp, out / "manifest.json")
        return out / "manifest.json"
    except BaseException:
        shutil.rmtree(out)
        raise


def load_mechanism_tasks(manifest, split="val"):
    """Verify checksums, exact labels and held-out composition isolation; return (metadata, rows)."""
    if split not in ("train", "val"):
        raise ValueError("mechanism split must be train or val")
    path = _manifest_path(manifest)
    manifest_hash(path)
    meta = json.loads(path.read_text())
    if meta.get("generator_version") != MECHANISM_VERSION or meta.get("format_version") != 1:
        raise ValueError("unsupported mechanism generator version")
    try:
        counts, seed = meta["examples_per_task"], meta["seed"]
        _mechanism_bounds(seed, counts["train"], counts["val"])
        parts = _mechanism_partitions(seed)
        declared = meta["composition_splits"]
        if set(meta["files"]) != {"train.jsonl", "val.jsonl"} or meta.get("counts_are_per_task") is not True:
            raise ValueError("invalid mechanism files/count semantics")
        loaded, ids = {}, set()
        for name in ("train", "val"):
            art = path.with_name(f"{name}.jsonl")
            info = meta["files"][art.name]
            if art.stat().st_size != info["bytes"] or _sha(art) != info["sha256"]:
                raise ValueError(f"mechanism artifact checksum/size mismatch: {art.name}")
            rows = []
            for line in art.read_text().splitlines():
                if len(rows) >= counts[name] * len(_MECHANISM_TASKS):
                    raise ValueError("mechanism rows exceed declared bounded counts")
                r = json.loads(line)
                task = r["task"]
                if task not in _MECHANISM_TASKS or r["split"] != name:
                    raise ValueError("invalid mechanism task/split")
                if task == "boolean_hierarchy":
                    comp, inst = tuple(r["operators"]), tuple(r["bits"])
                else:
                    pairs = r["key_values"]
                    if [p[0] for p in pairs] != list(_MECHANISM_KEYS):
                        raise ValueError("invalid retrieval keys")
                    comp, inst = tuple(p[1] for p in pairs), r["query"]
                if comp not in parts[task][name]:
                    raise ValueError("mechanism composition violates held-out partition")
                if r != _mechanism_row(task, name, comp, inst) or r["id"] in ids:
                    raise ValueError("invalid mechanism exact label/prompt/identity or duplicate row")
                ids.add(r["id"])
                rows.append(r)
            for task in _MECHANISM_TASKS:
                tr = [r for r in rows if r["task"] == task]
                if len(tr) != counts[name]:
                    raise ValueError("mechanism task count mismatch")
                comps = sorted({r["composition_id"] for r in tr})
                if declared[task][name] != comps:
                    raise ValueError("mechanism declared composition lists mismatch")
                if task == "boolean_hierarchy" and (sum(r["answer"] == " 1" for r in tr) * 2 != counts[name]
                                                    or len(comps) != 4):
                    raise ValueError("Boolean labels unbalanced or composition coverage missing")
            loaded[name] = rows
        for task in _MECHANISM_TASKS:
            if set(declared[task]["train"]) & set(declared[task]["val"]):
                raise ValueError("mechanism split composition overlap")
        return meta, loaded[split]
    except (KeyError, TypeError, IndexError) as e:
        raise ValueError(f"invalid mechanism metadata/rows: {e}") from e


def audit_mechanism_training(task_manifest, training_manifest) -> dict:
    """Which task compositions the declared train/calibration corpus exposes (exact text hashes),
    and whether the corpus is exactly the benchmark's train.jsonl with no validation overlap."""
    task_path, train_path = _manifest_path(task_manifest), _manifest_path(training_manifest)
    task_meta, train_rows = load_mechanism_tasks(task_path, "train")
    _, val_rows = load_mechanism_tasks(task_path, "val")
    task_hash, train_hash = manifest_hash(task_path), manifest_hash(train_path)
    training = json.loads(train_path.read_text())
    docs_path = train_path.with_name("documents.jsonl")
    if _sha(docs_path) != training.get("artifacts", {}).get("documents.jsonl"):
        raise ValueError("training document metadata checksum mismatch")
    source = training.get("source", {})
    source_matches = source.get("kind") == "jsonl" and source.get("sha256") == task_meta["files"]["train.jsonl"]["sha256"]
    by_hash = {}
    for split, rows in (("train", train_rows), ("val", val_rows)):
        for r in rows:
            for h in {_digest(r["text"]), _digest(r["text"].replace("\r\n", "\n").replace("\r", "\n"))}:
                by_hash.setdefault(h, []).append((split, r))
    exposed = {s: {t: set() for t in _MECHANISM_TASKS} for s in ("train", "calibration")}
    overlap = {t: set() for t in _MECHANISM_TASKS}
    train_ids = {r["id"] for r in train_rows}
    matched, unmatched = set(), 0
    total = 0
    for line in docs_path.read_text().splitlines():
        doc = json.loads(line)
        if doc["split"] not in exposed:
            continue
        total += 1
        hit = False
        for field in ("content_sha256", "processed_sha256"):
            for split, r in by_hash.get(doc[field].lower(), []):
                exposed[doc["split"]][r["task"]].add(r["composition_id"])
                if split == "val":
                    overlap[r["task"]].add(r["composition_id"])
                elif r["id"] == doc["id"]:
                    hit = True
        if hit and doc["id"] in train_ids:
            matched.add(doc["id"])
        else:
            unmatched += 1
    has_overlap = any(overlap.values())
    verified = bool(source_matches and not unmatched and total and not has_overlap)
    return {"verified": verified, "status": "overlap" if has_overlap else ("verified" if verified else "unknown"),
            "benchmark_manifest_hash": task_hash, "training_manifest_hash": train_hash,
            "source_matches_benchmark_train_sha256": source_matches,
            "coverage": {"declared_train_rows": len(train_rows), "train_calibration_documents": total,
                         "matched_declared_train_rows": len(matched), "unmatched_documents": unmatched,
                         "fraction": len(matched) / len(train_rows)},
            "exposed_compositions": {s: {t: sorted(v) for t, v in ts.items()} for s, ts in exposed.items()},
            "validation_composition_overlap": {t: sorted(v) for t, v in overlap.items()},
            "has_validation_overlap": has_overlap,
            "scope": "declared checksum-bound train/calibration corpus metadata only; exact whole-document text equality"}
