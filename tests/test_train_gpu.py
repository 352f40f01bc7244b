"""The serial trainer on CUDA: fused sm_100a path, exact interrupted replay, first update
consistent with the fp32 CPU trajectory."""
import copy
import json

import pytest
import torch

from helpers import FixtureTokenizer, state
from tensor_train_ing_b200 import train as trainer
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.data import prepare_data

pytestmark = pytest.mark.gpu


@pytest.fixture
def gpu_config(tmp_path, monkeypatch):
    """A 2-layer model the fused kernels cover, over a character-tokenized fixture dataset.  The
    trainer keeps test-only tokenizers on the CPU; this fixture lifts that for its own data."""
    text = "the quick brown fox jumps over the lazy dog; pack my box with five dozen liquor jugs. "
    source = tmp_path / "source.jsonl"
    source.write_text("".join(json.dumps({"id": str(i), "text": (text * 5)[i % 37:]}) + "\n" for i in range(80)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=source, revision="offline-v1",
                            tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .9, "val": 0., "test": 0., "calibration": .1})
    check = trainer._check_tokenizer
    monkeypatch.setattr(trainer, "_check_tokenizer",
                        lambda tok, named, dev: check({k: v for k, v in tok.items() if k != "test_only"}, named, dev))
    return Config(model=ModelConfig(layers=2, d_model=128, heads=2, d_key=64, d_value=64, d_mlp=256,
                                    vocab_size=50257, padded_vocab=50304),
                  train=TrainConfig(compile=False, global_prediction_tokens_per_update=600, rung_total_tokens=20_000,
                                    lr=3e-3),
                  raw={"data": {"manifest": str(manifest), "context": 128, "micro_batch_size": 2,
                                "calibration_tokens": 64},
                       "project": {"dry_run": False, "gpu_hourly_rate_usd": 1.0,
                                   "spend_ledger": str(tmp_path / "spend.json")}})


def test_cuda_training_uses_fused_path_and_replays_exactly(gpu_config, tmp_path):
    full = trainer.train_run(gpu_config, tmp_path / "full", max_steps=4, max_seconds=600, device="cuda")
    first = trainer.train_run(gpu_config, tmp_path / "a", max_steps=2, max_seconds=600, device="cuda")
    resumed = trainer.train_run(gpu_config, tmp_path / "b", max_steps=2, max_seconds=600, device="cuda",
                                resume=first["checkpoint"])
    assert full["progress"]["steps"] == resumed["progress"]["steps"] == 4
    rows = [json.loads(x) for x in (tmp_path / "full" / "metrics.jsonl").read_text().splitlines()]
    assert all(r["prediction_tokens"] == 600 and r["microbatches"] >= 2 for r in rows)
    assert all(torch.isfinite(torch.tensor([r["loss"], r["grad_norm"]])).all() for r in rows)
    assert rows[-1]["loss"] < rows[0]["loss"]
    a, b = state(tmp_path / "full" / "final"), state(tmp_path / "b" / "final")
    assert a["extra"]["runtime"]["fused_sm100a_path"] is True
    for k, v in a["model"].items():
        assert torch.equal(v, b["model"][k]), k
    tail = [json.loads(x) for x in (tmp_path / "b" / "metrics.jsonl").read_text().splitlines()]
    assert [r["loss"] for r in tail] == [r["loss"] for r in rows[2:]]


def test_cuda_first_update_agrees_with_cpu(gpu_config, tmp_path):
    """Same initial weights and batches: the bf16 fused path's first loss and gradient norm are the
    fp32 CPU trajectory's to within bf16 rounding."""
    cpu_cfg = copy.deepcopy(gpu_config)
    cpu_cfg.train.bf16_compute = False
    cpu_cfg.raw["project"]["gpu_hourly_rate_usd"] = 0
    cpu = trainer.train_run(cpu_cfg, tmp_path / "cpu", max_steps=1, max_seconds=600, device="cpu")
    gpu = trainer.train_run(gpu_config, tmp_path / "gpu", max_steps=1, max_seconds=600, device="cuda")
    c, g = cpu["history"][0], gpu["history"][0]
    assert c["batch_hashes"] == g["batch_hashes"]
    assert abs(g["loss"] - c["loss"]) <= 1e-2 * c["loss"]
    assert abs(g["grad_norm"] - c["grad_norm"]) <= 5e-2 * c["grad_norm"]
