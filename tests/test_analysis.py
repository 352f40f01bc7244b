"""Mechanistic analysis on CPU (tensor_train_ing_b200/analysis.py; reference tnlm/analysis.py):
spectral rank measures on known spectra, the restricted bilinear-MLP tensor reproducing the MLP,
operator classes and the report files of ``analyze``."""
import json
import math

import pytest
import torch

from tensor_train_ing_b200.analysis import analyze, entropy_rank, mlp_local_tensor, stable_rank
from tensor_train_ing_b200.config import ModelConfig
from tensor_train_ing_b200.models.model import TensorLM


def test_rank_measures_on_known_spectra():
    assert stable_rank(torch.tensor([3.0, 3.0, 3.0])) == pytest.approx(3.0)
    assert entropy_rank(torch.tensor([3.0, 3.0, 3.0])) == pytest.approx(3.0)
    assert stable_rank(torch.tensor([1.0, 0.0, 0.0])) == pytest.approx(1.0)
    assert entropy_rank(torch.tensor([1.0, 0.0, 0.0])) == pytest.approx(1.0)
    assert stable_rank(torch.tensor([2.0, -1.0])) == pytest.approx(1.25)  # sum s^2 / max s^2
    p = torch.tensor([2 / 3, 1 / 3])
    assert entropy_rank(torch.tensor([2.0, 1.0])) == pytest.approx(math.exp(-(p * p.log()).sum().item()))


def _probe(rows, T, seed):
    """(idx, doc ids, next-token targets) of one document per row."""
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, 40, (rows, T + 1), generator=g)
    return toks[:, :T], torch.zeros(rows, T, dtype=torch.long), toks[:, 1:]


def _model(dtype=torch.float32, **kw):
    torch.manual_seed(0)
    cfg = ModelConfig(layers=2, d_model=16, heads=2, d_key=8, d_value=8, d_mlp=24, vocab_size=40, padded_vocab=64, **kw)
    return TensorLM(cfg).to(dtype)


def test_restricted_mlp_tensor_reproduces_the_bilinear_mlp():
    model = _model(torch.float64)
    blk = model.blocks[0]
    U = torch.linalg.qr(torch.randn(16, 5, dtype=torch.float64)).Q
    z = torch.randn(7, 5, dtype=torch.float64)
    T = mlp_local_tensor(blk, U, fold_gain=False)
    za = torch.cat([z, torch.ones(7, 1, dtype=torch.float64)], 1) if T.shape[1] > 5 else z
    rec = torch.einsum("oab,na,nb->no", T, za, za)
    torch.testing.assert_close(rec, blk.mlp(z @ U.T), rtol=1e-10, atol=1e-12)
    assert torch.equal(T, T.transpose(1, 2))  # symmetrised


def test_analyze_writes_reports_and_leaves_the_model_unchanged(tmp_path):
    model = _model()
    model.train()
    before = {k: v.clone() for k, v in model.state_dict().items()}
    batches = [_probe(2, 12, seed) for seed in (1, 2)]
    result = analyze(model, batches, tmp_path / "ana")
    assert model.training  # mode restored
    for k, v in model.state_dict().items():
        assert torch.equal(v, before[k]), k
    assert result["operator_class"] == model.operator_audit()["class"]
    assert result["local_tensor"]["max_rel_err"] < 1e-5
    for row in result["local_tensor"]["per_layer"]:
        assert row["rel_err_gain_folded_on_probe"] < 1e-4
    assert set(result["normalizer_scopes"]) and all(isinstance(s, str) for s in result["normalizer_scopes"].values())
    for name in result["files"]:
        assert (tmp_path / "ana" / name).exists()
    assert json.loads((tmp_path / "ana" / "analysis.json").read_text())["operator_class"] == result["operator_class"]
    with pytest.raises(ValueError):
        analyze(model, [], tmp_path / "empty")


def test_swiglu_layers_are_skipped_by_the_local_tensor_check(tmp_path):
    model = _model(mlp="swiglu")
    batches = [_probe(1, 8, 3)]
    result = analyze(model, batches, tmp_path / "ana")
    assert all(row.get("skipped") for row in result["local_tensor"]["per_layer"])
    assert result["operator_class"] == "G"
