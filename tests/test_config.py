"""The configuration schema (CPU): unknown keys are rejected, extra sections are kept verbatim,
values validate, and anything but a mapping is refused rather than reinterpreted (a sweep candidate
list once loaded as a default configuration)."""
import pytest
import yaml

from tensor_train_ing_b200.config import Config, ModelConfig


def test_yaml_round_trip_keeps_every_section(tmp_path):
    doc = {"model": {"layers": 3, "d_model": 64, "heads": 4, "d_key": 16, "d_value": 16, "d_mlp": 96},
           "train": {"optimizer": "muon", "lr": 0.006, "aux_adamw_lr": 4.5e-4},
           "data": {"context": 128, "micro_batch_size": 2}, "project": {"dry_run": True},
           "evaluation": {"bootstrap_samples": 10}, "b200": {"anything": [1, 2]}}
    path = tmp_path / "run.yaml"
    path.write_text(yaml.safe_dump(doc))
    cfg = Config.from_yaml(str(path))
    assert cfg.model.layers == 3 and cfg.train.optimizer == "muon" and cfg.train.lr == 0.006
    assert cfg.raw["b200"] == {"anything": [1, 2]} and cfg.raw["data"]["context"] == 128
    again = Config.from_dict(cfg.to_dict())
    assert again.model == cfg.model and again.train == cfg.train


def test_unknown_keys_and_invalid_values_are_rejected():
    with pytest.raises(ValueError, match="unknown ModelConfig keys"):
        Config.from_dict({"model": {"layerz": 2}})
    with pytest.raises(ValueError, match="unknown TrainConfig keys"):
        Config.from_dict({"train": {"learning_rate": 1.0}})
    with pytest.raises(AssertionError):
        ModelConfig(normalization="layernorm")
    with pytest.raises(ValueError):
        ModelConfig(normalization="lagged")  # the lagged package needs the lagged final norm


def test_anything_but_a_mapping_is_refused(tmp_path):
    candidates = tmp_path / "candidates.yaml"
    candidates.write_text(yaml.safe_dump([{"name": "a", "overrides": {}}, {"name": "b", "overrides": {}}]))
    with pytest.raises(ValueError, match="mapping"):
        Config.from_yaml(str(candidates))
    with pytest.raises(ValueError, match="ModelConfig section must be a mapping"):
        Config.from_dict({"model": [["layers", 2]]})
    empty = tmp_path / "empty.yaml"
    empty.write_text("")
    assert Config.from_yaml(str(empty)).model == ModelConfig()  # an empty file is the defaults
