"""The ``train.deterministic`` policy (``runtime.deterministic_execution`` around every training entry
point) on CPU:

* the policy holds for the run only: torch's deterministic-algorithm flag, the cuDNN switches and
  ``CUBLAS_WORKSPACE_CONFIG`` are back to their earlier values afterwards, also after a failure;
* the run records the policy it trained under; a malformed value is refused before anything is
  written; a dry run changes no process state;
* a deterministic CUDA run asked for after CUDA was initialised without the cuBLAS workspace setting
  is refused before any flag changes (that setting only takes effect before CUDA starts), and an
  existing ``:4096:8`` or ``:16:8`` setting is accepted and kept.
"""
import copy
import os

import pytest
import torch

from tensor_train_ing_b200 import runtime
from tensor_train_ing_b200.runtime import deterministic_execution, determinism_metadata
from tensor_train_ing_b200.train import train_run


def _flags():
    meta = determinism_metadata()
    meta.pop("scope")
    return meta


@pytest.fixture
def clean_env(monkeypatch):
    monkeypatch.delenv("CUBLAS_WORKSPACE_CONFIG", raising=False)
    torch.use_deterministic_algorithms(False)
    yield
    torch.use_deterministic_algorithms(False)


def test_the_policy_is_scoped_to_the_body_and_restored_after_a_failure(clean_env):
    before = _flags()
    with deterministic_execution(True, device="cpu"):
        inside = _flags()
        assert inside["algorithms_enabled"] and inside["cudnn_deterministic"] and not inside["cudnn_benchmark"]
        assert os.environ["CUBLAS_WORKSPACE_CONFIG"] == ":4096:8"
    assert _flags() == before and "CUBLAS_WORKSPACE_CONFIG" not in os.environ
    with pytest.raises(KeyError):
        with deterministic_execution(True, device="cpu"):
            raise KeyError("a failure inside the run")
    assert _flags() == before
    with deterministic_execution(False, device="cpu"):
        assert not torch.are_deterministic_algorithms_enabled()
    assert _flags() == before
    with pytest.raises(ValueError, match="Boolean"):
        with deterministic_execution("yes", device="cpu"):
            pass


def test_late_cuda_setup_is_refused_without_changing_anything(clean_env, monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_initialized", lambda: True)
    before = _flags()
    with pytest.raises(RuntimeError, match="CUBLAS_WORKSPACE_CONFIG"):
        with deterministic_execution(True, device="cuda"):
            pass
    assert _flags() == before and "CUBLAS_WORKSPACE_CONFIG" not in os.environ
    with deterministic_execution(False, device="cuda"):  # nondeterministic runs need nothing
        pass


@pytest.mark.parametrize("workspace", [":4096:8", ":16:8"])
def test_an_existing_workspace_setting_is_used_and_kept(clean_env, monkeypatch, workspace):
    monkeypatch.setenv("CUBLAS_WORKSPACE_CONFIG", workspace)
    monkeypatch.setattr(torch.cuda, "is_initialized", lambda: True)
    with deterministic_execution(True, device="cuda"):
        assert torch.are_deterministic_algorithms_enabled()
        assert os.environ["CUBLAS_WORKSPACE_CONFIG"] == workspace
    assert not torch.are_deterministic_algorithms_enabled()
    assert os.environ["CUBLAS_WORKSPACE_CONFIG"] == workspace


def test_training_records_its_policy_and_restores_the_process(config, tmp_path, clean_env):
    cfg = copy.deepcopy(config)
    cfg.train.deterministic = True
    before = _flags()
    result = train_run(cfg, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    recorded = result["runtime"]["determinism"]
    assert recorded["algorithms_enabled"] is True and recorded["cublas_workspace_config"] == ":4096:8"
    assert _flags() == before


def test_a_malformed_policy_is_refused_before_any_write(config, tmp_path, clean_env):
    cfg = copy.deepcopy(config)
    cfg.train.deterministic = "true"
    with pytest.raises(ValueError, match="Boolean"):
        train_run(cfg, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    assert not (tmp_path / "run").exists()


def test_a_dry_run_changes_no_process_state(config, tmp_path, clean_env, monkeypatch):
    cfg = copy.deepcopy(config)
    cfg.train.deterministic = True
    cfg.raw.setdefault("project", {})["dry_run"] = True
    calls = []
    monkeypatch.setattr(runtime, "deterministic_execution", lambda *a, **k: calls.append(a))
    before = _flags()
    train_run(cfg, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    assert _flags() == before and not calls and not (tmp_path / "run").exists()
