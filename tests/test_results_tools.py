"""Experiment-result tools (``runbook/results.py``) on CPU: the LR-optimum fit recovers a planted
optimum and its power law, the contamination check finds near-duplicated validation documents, the
evaluated-state listing respects age and keep rules, and the export writes a weight-free, thinned,
idempotent mirror."""
import json
import math
import os
import time

import pytest

from helpers import FixtureTokenizer
from tensor_train_ing_b200.data import prepare_data
from tensor_train_ing_b200.runbook import results

PATTERN = r"w(?P<group>\d+)_lr(?P<lr>[0-9.e-]+)"


def _report(runs, name, ce, lr=None):
    path = runs / name / "evaluation" / "evaluation.json"
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"ce": ce, "training_descriptor": {"lr": lr}}))
    return path


def _planted(g, lr):
    """CE parabola in log(lr), optimum 0.004 * (g / 256) ** -0.5."""
    opt = 0.004 * (g / 256) ** -0.5
    return 3.0 + 0.1 * (math.log(lr) - math.log(opt)) ** 2


def test_lr_optimum_recovers_the_planted_optimum_and_power_law(tmp_path):
    runs = tmp_path / "runs"
    for g in (256, 1024):
        for lr in (0.001, 0.002, 0.004, 0.008, 0.016):
            _report(runs, f"w{g}_lr{lr}", _planted(g, lr))
    _report(runs, "unrelated_name", 1.0)
    fits = results.fit_lr_optimum(results.collect_lr_points(runs, PATTERN))
    assert set(fits) == {256, 1024}
    for g, f in fits.items():
        assert f["optimum"] == pytest.approx(0.004 * (g / 256) ** -0.5, rel=1e-6)
        assert f["optimum_ce"] == pytest.approx(3.0, abs=1e-9) and f["interior"] and not f["flat"]
        assert f["next_lr"] is None
    law = results.optimum_power_law(fits)
    assert law["slope"] == pytest.approx(-0.5, abs=1e-6) and law["k"] > 0


def test_lr_optimum_edges_flat_duplicates_and_exclusion(tmp_path):
    runs = tmp_path / "runs"
    for lr in (0.001, 0.002, 0.004):  # still falling at the largest rate
        _report(runs, f"w64_lr{lr}", 3.0 - lr)
    for lr in (0.001, 0.002, 0.004):  # spread far below the evaluation noise
        _report(runs, f"w128_lr{lr}", 3.0 + 1e-4 * (lr * 1000 - 2) ** 2)
    _report(runs, "w32_lr0.001", 3.1)
    _report(runs, "w32_lr0.002", 3.0)
    old = _report(runs / "old", "w16_lr0.001", 9.0)
    os.utime(old, (time.time() - 100, time.time() - 100))
    _report(runs / "new", "w16_lr0.001", 4.0)  # the newer evaluation of the same point wins
    _report(runs / "skip", "w16_lr0.002", 0.0)
    fits = results.fit_lr_optimum(results.collect_lr_points(runs, PATTERN, exclude=r"^skip/"))
    assert fits[64]["next_lr"] == pytest.approx(0.008) and not fits[64]["interior"]
    assert fits[128]["flat"] and results.optimum_power_law(fits) is None
    assert fits[32]["optimum"] is None and fits[32]["next_lr"] == pytest.approx(0.004)
    assert fits[16]["ce"] == [4.0]
    named = tmp_path / "named"
    _report(named, "w8_x2", 3.0, lr=0.006)  # a grid name holding a multiplier: the rate is the descriptor's
    assert results.collect_lr_points(named, r"w(?P<group>\d+)_x\d+", descriptor_lr=True) == {8: {0.006: 3.0}}


def test_contamination_finds_near_duplicates_of_validation_documents(tmp_path):
    import random
    rngs = [random.Random(i) for i in range(40)]
    texts = [f"document {i}: " + "".join(r.choice("abcdefghijklmnopqrstuvwxyz") for _ in range(80))
             for i, r in enumerate(rngs)]
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"d{i}", "text": t}) + "\n" for i, t in enumerate(texts)))
    manifest = prepare_data(tmp_path / "val", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .5, "val": .5, "test": 0., "calibration": 0.})
    val_ids = [json.loads(x)["id"] for x in (tmp_path / "val" / "documents.jsonl").read_text().splitlines()
               if json.loads(x)["split"] == "val"]
    copied = val_ids[:3]
    train_texts = [f"other text {i} " + "xyz" * 20 for i in range(10)]
    train_texts += [f"header boilerplate -- {texts[int(i[1:])]} -- footer" for i in copied]
    src2 = tmp_path / "src2.jsonl"
    src2.write_text("".join(json.dumps({"id": f"t{i}", "text": t}) + "\n" for i, t in enumerate(train_texts)))
    prepare_data(tmp_path / "train", source_jsonl=src2, revision="offline-v1", tokenizer=FixtureTokenizer(),
                 split_fractions={"train": 1., "val": 0., "test": 0., "calibration": 0.})
    report = results.contamination(tmp_path / "train", tmp_path / "val", n=13)
    flagged = {d["id"] for d in report["flagged"]}
    assert flagged == set(copied)
    # every window but those reaching the document's end-of-text token, which the copy lacks
    assert all(d["overlap"] > 0.95 for d in report["flagged"])
    assert report["validation_documents"] == len(val_ids)
    assert results.main(["contamination", "--train", str(tmp_path / "train"), "--val", str(tmp_path / "val")]) == 1


def test_window_hashes_match_windows():
    import numpy as np
    t = np.array([5, 1, 2, 5, 1, 2, 9], dtype=np.uint16)
    h = results.window_hashes(t, 3)
    assert len(h) == 5 and h[0] == h[3] and len(set(h.tolist())) == 4
    assert len(results.window_hashes(t[:2], 3)) == 0


def test_evaluated_states_respect_age_and_keep(tmp_path):
    runs = tmp_path / "runs"
    evaluated = runs / "a" / "parent" / "milestone-8" / "state.pt"
    fresh = runs / "a" / "parent" / "final" / "state.pt"
    kept = runs / "keepme" / "final" / "state.pt"
    pending = runs / "b" / "final" / "state.pt"
    for p in (evaluated, fresh, kept, pending):
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_bytes(b"x" * 100)
    for run in (runs / "a", runs / "keepme"):
        (run / "evaluation").mkdir(parents=True)
        (run / "evaluation" / "evaluation.json").write_text("{}")
    now = time.time()
    for p in (evaluated, kept, pending):
        os.utime(p, (now - 3600, now - 3600))
    found = results.evaluated_states(runs, min_age_min=30, keep=["keepme"], now=now)
    assert [f["path"] for f in found] == [str(evaluated)] and found[0]["bytes"] == 100
    assert evaluated.exists()  # nothing deleted


def test_export_is_thinned_weight_free_and_idempotent(tmp_path):
    runs, out = tmp_path / "runs", tmp_path / "out"
    run = runs / "cand" / "parent"
    run.mkdir(parents=True)
    rows = [{"step": i + 1, "tokens": 10 * (i + 1), "loss": 5.0 - i / 1000, "lr": 0.01, "grad_norm": 1.0,
             "seconds": 0.1} for i in range(1000)]
    rows[500]["qk_clip"] = {"clipped_heads": 2}
    (run / "metrics.jsonl").write_text("".join(json.dumps(r) + "\n" for r in rows))
    (run / "final").mkdir()
    (run / "final" / "state.pt").write_bytes(b"weights")
    ev = runs / "cand" / "evaluation"
    ev.mkdir()
    (ev / "evaluation.json").write_text(json.dumps({"ce": 3.2, "prediction_tokens": 99, "uncertainty": {},
                                                    "training_descriptor": {"lr": 0.01}, "bulky": "x" * 1000}))
    first = results.export_results(runs, out, max_rows=100)
    curve = json.loads((out / "cand" / "parent" / "curve.json").read_text())
    assert len(curve["rows"]) <= 101 and curve["rows"][-1]["step"] == 1000 and curve["rows"][0]["step"] == 1
    assert curve["logged_rows"] == 1000 and curve["events"] == [{"step": 501, "qk_clip": {"clipped_heads": 2}}]
    summary = json.loads((out / "cand" / "evaluation" / "evaluation.json").read_text())
    assert summary["ce"] == 3.2 and "bulky" not in summary
    assert not list(out.rglob("*.pt")) and len(first["written"]) == 2
    again = results.export_results(runs, out, max_rows=100)
    assert again["written"] == [] and len(again["unchanged"]) == 2


def test_the_command_line_prints_json_for_every_tool(tmp_path, capsys):
    runs = tmp_path / "runs"
    for lr in (0.001, 0.002, 0.004):
        _report(runs, f"w64_lr{lr}", _planted(64, lr))
    assert results.main(["lr-optimum", str(runs), "--pattern", PATTERN]) == 0
    fit = json.loads(capsys.readouterr().out)
    assert fit["groups"]["64"]["optimum"] == pytest.approx(0.008, rel=1e-6) and fit["power_law"] is None
    assert results.main(["states", str(runs), "--min-age-min", "0"]) == 0
    assert json.loads(capsys.readouterr().out) == {"states": [], "total_bytes": 0}
    assert results.main(["export", str(runs), str(tmp_path / "out")]) == 0
    assert len(json.loads(capsys.readouterr().out)["written"]) == 3
