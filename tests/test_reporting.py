"""Run summaries, batched evaluation comparisons, paired-seed validation checks, the token payload
format and ordered tokenization (CPU; the reference covers the same modules in
tests/test_reporting_schedule.py, test_comparison_batch.py, test_replication.py, test_token_format.py
and test_data.py)."""
import json

import numpy as np
import pytest
import torch

from helpers import FixtureTokenizer
from tensor_train_ing_b200.checkpoint import save_checkpoint
from tensor_train_ing_b200.comparison_batch import compare_evaluation_pairs
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.data import manifest_hash, prepare_data
from tensor_train_ing_b200.data_preparation import batches, encode_batch, ordered_tokenization, token_array
from tensor_train_ing_b200.evaluate import evaluate_checkpoint
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.replication import compare_seed_pairs
from tensor_train_ing_b200.reporting import summarize_runs
from tensor_train_ing_b200.runtime import full_config
from tensor_train_ing_b200.token_format import read_split_tokens
from tensor_train_ing_b200.train import train_run


# ------------------------------------------------------------------------------ run summaries
def test_summarize_two_runs_writes_table_csv_and_three_svg_plots(config, tmp_path):
    runs = []
    for name, lr in (("lr-a", 0.01), ("lr-b", 0.02)):
        config.train.lr = lr
        train_run(config, tmp_path / name, max_steps=3, max_seconds=120, device="cpu")
        runs.append(tmp_path / name)
    out = summarize_runs(runs, tmp_path / "summary", max_plot_points=2)
    assert out["runs"] == 2
    assert out["artifacts"] == ["comparison.csv", "comparison.json", "loss-vs-cost.svg", "loss-vs-time.svg",
                                "loss-vs-tokens.svg"]
    bundle = json.loads((tmp_path / "summary" / "comparison.json").read_text())
    assert bundle["automatic_ranking_eligible"] is False
    assert [r["configured_lr"] for r in bundle["runs"]] == [0.01, 0.02]
    for row in bundle["runs"]:
        assert row["run_prediction_tokens"] == row["global_prediction_tokens"] > 0
        assert row["final_training_ce"] > 0
    # the curve is thinned to at most max_plot_points (+ the last point) but keeps both ends
    curve = bundle["curves"][0]
    assert curve["original_metric_points"] == 3 and 2 <= len(curve["points"]) <= 3
    assert curve["points"][-1]["step"] == 3
    header = (tmp_path / "summary" / "comparison.csv").read_text().splitlines()[0]
    assert header.startswith("run,operator_class,normalization,optimizer,configured_lr")
    svg = (tmp_path / "summary" / "loss-vs-tokens.svg").read_text()
    assert svg.count("<polyline") == 2 and "lr-a" in svg and "lr-b" in svg
    with pytest.raises(FileExistsError):  # outputs are never overwritten
        summarize_runs(runs, tmp_path / "summary")
    with pytest.raises(ValueError):
        summarize_runs(runs, tmp_path / "again", max_plot_points=1)


def test_summary_refuses_an_unfinished_run(config, tmp_path):
    train_run(config, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    result = json.loads((tmp_path / "run" / "result.json").read_text())
    ledger_path = result["spend_ledger"]
    ledger = json.loads(open(ledger_path).read())
    ledger["runs"][result["run_id"]]["status"] = "running"
    open(ledger_path, "w").write(json.dumps(ledger))
    with pytest.raises(ValueError, match="unfinished"):
        summarize_runs([tmp_path / "run"], tmp_path / "summary")


# --------------------------------------------------------------------- evaluation comparisons
@pytest.fixture
def reports(tmp_path):
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 2}) + "\n" for i in range(40)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    cfg = Config(model=ModelConfig(layers=1, d_model=8, heads=1, d_key=4, d_value=4, d_mlp=12, padded_vocab=50257),
                 train=TrainConfig(compile=False, bf16_compute=False),
                 raw={"data": {"manifest": str(manifest), "context": 16},
                      "project": {"dry_run": False, "gpu_hourly_rate_usd": 0,
                                  "spend_ledger": str(tmp_path / "spend.json")}})
    out = {}
    for name, seed in (("a", 1), ("b", 2), ("c", 3)):
        torch.manual_seed(seed)
        model = TensorLM(cfg.model)
        save_checkpoint(tmp_path / f"ckpt-{name}", model, None, None, config=full_config(cfg),
                        progress={"steps": 0, "tokens": 0}, manifest_hash=manifest_hash(manifest))
        r = evaluate_checkpoint(cfg, tmp_path / f"ckpt-{name}", tmp_path / f"eval-{name}", max_seconds=120,
                                device="cpu", bootstrap_samples=10)
        out[name] = (tmp_path / f"eval-{name}" / "evaluation.json", r)
    return out, tmp_path


def test_batched_comparisons_bind_each_report_once_and_keep_pair_order(reports):
    reps, tmp = reports
    pairs = [{"name": "a-vs-b", "left": str(reps["a"][0]), "right": str(reps["b"][0])},
             {"name": "a-vs-c", "left": str(reps["a"][0]), "right": str(reps["c"][0])}]
    out = compare_evaluation_pairs(pairs, tmp / "cmp", bootstrap_samples=20, seed=3)
    assert [p["name"] for p in out["pairs"]] == ["a-vs-b", "a-vs-c"]
    assert len(out["inputs"]) == 3  # report a is read (and hashed) once
    for p, other in zip(out["pairs"], ("b", "c")):
        assert p["result"]["delta_ce_right_minus_left"] == pytest.approx(reps[other][1]["ce"] - reps["a"][1]["ce"],
                                                                         rel=1e-9, abs=1e-12)
    written = json.loads((tmp / "cmp" / "comparisons.json").read_text())
    assert written["automatic_ranking_eligible"] is False and written["seed"] == 3
    with pytest.raises(FileExistsError):
        compare_evaluation_pairs(pairs, tmp / "cmp")
    for bad in ([], [{"name": "x", "left": str(reps["a"][0])}],
                [pairs[0], dict(pairs[1], name="a-vs-b")]):  # empty, missing side, duplicate name
        with pytest.raises(ValueError):
            compare_evaluation_pairs(bad, tmp / "bad")
    with pytest.raises(ValueError):
        compare_evaluation_pairs(pairs, tmp / "bad", bootstrap_samples=-1)


def test_paired_seed_validation_rejects_malformed_requests(reports):
    reps, tmp = reports
    a, b = str(reps["a"][0]), str(reps["b"][0])
    one = [{"seed": 1, "left": a, "right": b}]
    with pytest.raises(ValueError, match="two"):
        compare_seed_pairs(one, tmp / "r", allowed_between_dimensions=[])
    two = one + [{"seed": 2, "left": a, "right": b}]
    with pytest.raises(ValueError, match="seed cannot"):
        compare_seed_pairs(two, tmp / "r", allowed_between_dimensions=["seed"])
    with pytest.raises(ValueError, match="unique"):
        compare_seed_pairs(two, tmp / "r", allowed_between_dimensions=["lr", "lr"])
    with pytest.raises(ValueError, match="unique nonnegative"):
        compare_seed_pairs([{"seed": -1, "left": a, "right": b}] + one, tmp / "r", allowed_between_dimensions=[])
    with pytest.raises(ValueError, match="exactly seed"):
        compare_seed_pairs([{"seed": 1, "left": a}] + one, tmp / "r", allowed_between_dimensions=[])
    # untrained checkpoints carry no complete configuration evidence with the declared seed
    with pytest.raises(ValueError):
        compare_seed_pairs(two, tmp / "r", allowed_between_dimensions=[])
    assert not (tmp / "r").exists()


# ---------------------------------------------------------------- token format and tokenization
def test_split_tokens_are_little_endian_int32_and_read_only(tmp_path):
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": str(i), "text": "abc" * (i + 1)}) + "\n" for i in range(10)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .8, "val": .2, "test": 0., "calibration": 0.})
    root = manifest.parent if manifest.is_file() else manifest
    train = read_split_tokens(root, "train")
    assert train.dtype == np.dtype("<i4") and len(train) > 0 and not train.flags.writeable
    raw = (root / "train.tokens.bin").read_bytes()
    assert np.array_equal(np.frombuffer(raw, dtype="<i4"), np.asarray(train))
    empty = read_split_tokens(root, "test")
    assert len(empty) == 0 and not empty.flags.writeable
    with pytest.raises(ValueError):
        read_split_tokens(root, "holdout")
    (root / "val.tokens.bin").chmod(0o644)
    with open(root / "val.tokens.bin", "ab") as f:
        f.write(b"\x01")  # no longer a whole number of int32 tokens
    with pytest.raises(ValueError):
        read_split_tokens(root, "val")


def test_ordered_tokenization_is_independent_of_workers_and_batching():
    rows = [(f"d{i}", "line\r\n" * (i % 5) + "x" * (i * 37 % 300), i) for i in range(300)]
    serial = list(ordered_tokenization(rows, tokenizer=FixtureTokenizer(), workers=1, batch_bytes=1 << 20))
    pooled = list(ordered_tokenization(rows, tokenizer=FixtureTokenizer(), workers=3, batch_bytes=512))
    assert [r[0] for r in serial] == [r[0] for r in rows] == [r[0] for r in pooled]
    for s, p in zip(serial, pooled):
        assert s[1] == p[1] and np.array_equal(s[2], p[2]) and s[3] == p[3]
    # carriage returns are normalised before hashing and encoding
    (doc,) = encode_batch([("x", "a\r\nb\rc")], FixtureTokenizer())
    assert np.array_equal(doc[2], np.asarray([ord(c) for c in "a\nb\nc"]))
    assert token_array(doc[2]).dtype == np.dtype("<i4")
    sizes = [len(b) for b in batches([("d", "y" * 100)] * 10, 250)]
    assert sizes == [2, 2, 2, 2, 2]  # byte bound; a batch never exceeds it unless one document does
    assert [len(b) for b in batches([("d", "z")] * 300, 1 << 20)] == [128, 128, 44]  # 128 documents at most
    with pytest.raises(ValueError):
        list(ordered_tokenization(rows, tokenizer=FixtureTokenizer(), workers=0, batch_bytes=10))


def test_config_flattening_and_differences_are_type_exact():
    """Recorded configurations compare leaf by leaf on dot paths; an int and a float of equal value
    differ (a changed type is a changed configuration), an empty section is a leaf, and keys that
    would break the dot paths are refused."""
    from tensor_train_ing_b200.replication import config_differences, flatten_config
    tree = {"model": {"d_model": 8, "extra": {}}, "train": {"lr": 0.01, "seed": 1}}
    assert flatten_config(tree) == {"config.model.d_model": 8, "config.model.extra": {}, "config.train.lr": 0.01,
                                    "config.train.seed": 1}
    other = {"model": {"d_model": 8.0, "extra": {}}, "train": {"lr": 0.01, "seed": 2}}
    assert config_differences(tree, other) == ["config.model.d_model", "config.train.seed"]
    assert config_differences(tree, other, ignore=("config.train.seed",)) == ["config.model.d_model"]
    with pytest.raises(ValueError):
        config_differences(tree, {"model": {"d_model": 8}, "train": {"lr": 0.01, "seed": 1}})
    with pytest.raises(ValueError):
        flatten_config({"a.b": 1})
