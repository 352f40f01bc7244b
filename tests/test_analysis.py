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


def test_analytic_norm_jvp_matches_autograd_in_fp64():
    """The (group) RMSNorm Jacobian-vector product splits into a direct part delta/r and a radial part
    (the divisor's response); their sum equals autograd's JVP, and the radial part vanishes for a
    perturbation orthogonal to x within each group."""
    import torch

    from tensor_train_ing_b200.analysis import _analytic_jvp
    from tensor_train_ing_b200.models.normalization import GroupRMSNorm, RMSNorm
    torch.manual_seed(0)
    for norm in (RMSNorm(16, 1e-6).double(), GroupRMSNorm(16, 4).double()):
        with torch.no_grad():
            norm.weight.uniform_(0.5, 1.5)
        x = torch.randn(5, 16, dtype=torch.float64)
        delta = torch.randn(5, 16, dtype=torch.float64)
        direct, radial = _analytic_jvp(norm, x, delta)
        _, ref = torch.func.jvp(norm, (x,), (delta,))
        torch.testing.assert_close(direct + radial, ref, rtol=1e-10, atol=1e-12)
        groups = getattr(norm, "groups", 1)
        xs, ds = x.unflatten(-1, (groups, -1)), delta.unflatten(-1, (groups, -1))
        ortho = (ds - xs * (xs * ds).sum(-1, keepdim=True) / xs.square().sum(-1, keepdim=True)).flatten(-2)
        _, radial_ortho = _analytic_jvp(norm, x, ortho)
        assert float(radial_ortho.abs().max()) < 1e-12


def test_norm_gains_fold_lagged_and_refuse_a_mid_taper():
    """The fixed map a norm site folds into the adjacent linear maps: gamma for RMS, gamma over the
    frozen RMS for the lagged norm; a TaperRMS part-way through its gate has none."""
    import torch

    from tensor_train_ing_b200.analysis import gain, norm_scope
    from tensor_train_ing_b200.models.normalization import LaggedRMS, RMSNorm, TaperRMS
    rms = RMSNorm(8, 1e-6)
    assert torch.equal(gain(rms, 8, "cpu"), rms.weight.detach().float())
    assert norm_scope(rms) == "per-token RMS over all features"
    lag = LaggedRMS(8)
    with torch.no_grad():
        lag.mean_sq.fill_(4.0)
    expected = lag.weight.detach().float() / torch.sqrt(torch.tensor(4.0) + lag.eps)
    torch.testing.assert_close(gain(lag, 8, "cpu"), expected)
    taper = TaperRMS(8)
    with torch.no_grad():
        taper.gate.fill_(0.5)
    with pytest.raises(ValueError, match="no fixed map"):
        gain(taper, 8, "cpu")
    assert torch.equal(gain(torch.nn.Identity(), 8, "cpu"), torch.ones(8))
