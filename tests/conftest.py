import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")
    config.addinivalue_line("markers", "slow: multi-process or long-running")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def config(tmp_path):
    """Tiny CPU training config over a 20-document fixture dataset (context 4)."""
    import json

    import torch

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
    from tensor_train_ing_b200.data import prepare_data

    torch.set_num_threads(1)
    source = tmp_path / "source.jsonl"
    source.write_text("".join(json.dumps({"id": str(i), "text": "abcdefghijklm"}) + "\n" for i in range(20)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=source, revision="offline-v1",
                            tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .8, "val": 0., "test": 0., "calibration": .2})
    return Config(model=ModelConfig(layers=1, d_model=8, heads=1, d_key=4, d_value=4, d_mlp=12, padded_vocab=50257),
                  train=TrainConfig(compile=False, bf16_compute=False, global_prediction_tokens_per_update=7,
                                    rung_total_tokens=100, lr=.01),
                  raw={"data": {"manifest": str(manifest), "context": 4, "micro_batch_size": 1,
                                "calibration_tokens": 8},
                       "project": {"dry_run": False, "gpu_hourly_rate_usd": 0,
                                   "spend_ledger": str(tmp_path / "spend.json")}})
