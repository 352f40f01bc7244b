"""Full-state checkpoint format: integrity, atomic publish, preflight before mutation."""
import json

import pytest
import torch

from helpers import TINY_MODEL
from tensor_train_ing_b200.checkpoint import load_checkpoint, read_manifest, save_checkpoint
from tensor_train_ing_b200.config import ModelConfig, TrainConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.optim import MuonAdamW
from tensor_train_ing_b200.optim import make_optimizer as make_opt


def _model(seed=0):
    torch.manual_seed(seed)
    return TensorLM(ModelConfig(**TINY_MODEL))


def _save(path, model, optimizer=None, **kw):
    return save_checkpoint(path, model, optimizer, None, config={"model": {}}, progress={"steps": 0},
                           manifest_hash="m" * 64, **kw)


def _clone_state(m):
    return {k: v.clone() for k, v in m.state_dict().items()}


def test_full_state_roundtrip(tmp_path):
    m = _model(1)
    manifest = _save(tmp_path / "c", m)
    assert manifest["files"]["state.pt"]["bytes"] > 0
    other = _model(2)
    load_checkpoint(tmp_path / "c", other, restore_rng=False)
    for k, v in m.state_dict().items():
        assert torch.equal(v, other.state_dict()[k])


def test_reject_corrupt_incomplete_and_overwrite(tmp_path):
    m = _model()
    _save(tmp_path / "c", m)
    with pytest.raises(FileExistsError):
        _save(tmp_path / "c", m)
    state = tmp_path / "c" / "state.pt"
    raw = bytearray(state.read_bytes())
    raw[len(raw) // 2] ^= 0xFF
    state.write_bytes(bytes(raw))
    before = _clone_state(m)
    with pytest.raises(ValueError):
        load_checkpoint(tmp_path / "c", m)
    assert all(torch.equal(v, m.state_dict()[k]) for k, v in before.items())
    (tmp_path / "d").mkdir()
    with pytest.raises(ValueError):
        read_manifest(tmp_path / "d")


def test_shape_mismatch_preflight_does_not_mutate(tmp_path):
    _save(tmp_path / "c", _model())
    other = TensorLM(ModelConfig(**{**TINY_MODEL, "d_mlp": 64}))
    before = _clone_state(other)
    with pytest.raises(ValueError):
        load_checkpoint(tmp_path / "c", other, restore_rng=False)
    assert all(torch.equal(v, other.state_dict()[k]) for k, v in before.items())


def test_nonfinite_state_not_published(tmp_path):
    m = _model()
    with torch.no_grad():
        next(m.parameters()).view(-1)[0] = float("nan")
    with pytest.raises(Exception):
        _save(tmp_path / "c", m)
    assert not (tmp_path / "c").exists()
    assert not any(p.name.startswith(".c.tmp") for p in tmp_path.iterdir())


def test_failed_write_is_not_published(tmp_path, monkeypatch):
    import tensor_train_ing_b200.checkpoint as ck

    def boom(*a, **k):
        raise OSError("disk full")
    monkeypatch.setattr(ck.torch, "save", boom)
    with pytest.raises(OSError):
        _save(tmp_path / "c", _model())
    assert list(tmp_path.iterdir()) == []


def test_optimizer_state_roundtrip_and_mismatch(tmp_path):
    tc = TrainConfig(optimizer="muon", lr=0.01)
    m = _model()
    opt = make_opt(m, tc)
    assert isinstance(opt, MuonAdamW)
    idx = torch.randint(0, 97, (2, 5))
    _, loss = m(idx, targets=torch.roll(idx, -1, 1))
    loss.backward()
    opt.step()
    _save(tmp_path / "c", m, opt)
    m2 = _model(3)
    opt2 = make_opt(m2, tc)
    load_checkpoint(tmp_path / "c", m2, opt2, restore_rng=False)
    a, b = opt.state_dict(), opt2.state_dict()
    for part in ("muon", "adamw"):
        sa, sb = a[part]["state"], b[part]["state"]
        assert sa.keys() == sb.keys()
        for k in sa:
            for name, v in sa[k].items():
                assert torch.equal(torch.as_tensor(v), torch.as_tensor(sb[k][name]))
    adam = torch.optim.AdamW(m2.parameters())
    with pytest.raises(ValueError):
        load_checkpoint(tmp_path / "c", m2, adam, restore_rng=False)


def test_unfinished_stat_collection_rejected(tmp_path):
    m = TensorLM(ModelConfig(**{**TINY_MODEL, "normalization": "lagged", "final_normalization": "lagged"}))
    from tensor_train_ing_b200.models.normalization import lagged_modules
    norm = lagged_modules(m)[0]
    norm.collecting = True
    m(torch.randint(0, 97, (1, 4)))
    with pytest.raises(ValueError):
        _save(tmp_path / "c", m)


def test_identity_checks_refuse_another_dataset_or_config(tmp_path):
    """A checkpoint names the dataset (manifest hash) and the config it was trained with; loading it
    for another dataset or config is refused before any tensor is touched, and a validator may record
    a compatibility note instead."""
    m = _model(1)
    save_checkpoint(tmp_path / "c", m, None, None, config={"model": {"d_model": 32}, "train": {"lr": 0.1}},
                    progress={"steps": 3}, manifest_hash="a" * 64)
    target = _model(2)
    before = _clone_state(target)
    with pytest.raises(ValueError, match="Data manifest hash mismatch"):
        load_checkpoint(tmp_path / "c", target, expected_manifest_hash="b" * 64, restore_rng=False)
    with pytest.raises(ValueError, match="config mismatch"):
        load_checkpoint(tmp_path / "c", target, expected_config={"model": {"d_model": 64}, "train": {"lr": 0.1}},
                        restore_rng=False)
    for k, v in before.items():
        assert torch.equal(v, target.state_dict()[k])
    payload = load_checkpoint(tmp_path / "c", target, expected_manifest_hash="a" * 64,
                              config_validator=lambda saved: {"accepted_lr": saved["train"]["lr"]},
                              restore_rng=False)
    assert payload["config_compatibility"] == {"accepted_lr": 0.1} and payload["progress"]["steps"] == 3


def test_rng_streams_continue_after_a_restore(tmp_path):
    """The saved python / numpy / torch generator states are restored, so random draws after a
    resume are the draws an uninterrupted run makes."""
    import random

    import numpy as np
    m = _model(3)
    torch.manual_seed(123)
    random.seed(5)
    np.random.seed(7)
    _save(tmp_path / "c", m)
    want = (torch.rand(4), random.random(), np.random.rand(2))
    torch.manual_seed(0)
    random.seed(0)
    np.random.seed(0)
    load_checkpoint(tmp_path / "c", _model(4))
    got = (torch.rand(4), random.random(), np.random.rand(2))
    assert torch.equal(got[0], want[0]) and got[1] == want[1] and (got[2] == want[2]).all()


def test_sampler_cursor_resumes_the_batch_stream(tmp_path, config):
    """The data cursor travels with the checkpoint: a sampler restored from it yields the batches the
    original would have yielded next."""
    from tensor_train_ing_b200.data import PackedSampler
    manifest = config.raw["data"]["manifest"]
    s = PackedSampler(manifest, batch_size=2, context=4, seed=1)
    for _ in range(3):
        s.next_batch()
    m = _model(0)
    save_checkpoint(tmp_path / "c", m, None, s, config={"model": {}}, progress={"steps": 3},
                    manifest_hash=s.manifest_hash)
    expected = [s.next_batch() for _ in range(4)]
    fresh = PackedSampler(manifest, batch_size=2, context=4, seed=1)
    load_checkpoint(tmp_path / "c", _model(0), None, fresh, expected_manifest_hash=s.manifest_hash,
                    restore_rng=False)
    for want in expected:
        got = fresh.next_batch()
        assert all(torch.equal(a, b) for a, b in zip(got, want))
    other_seed = PackedSampler(manifest, batch_size=2, context=4, seed=2)
    with pytest.raises(ValueError):
        load_checkpoint(tmp_path / "c", _model(0), None, other_seed, restore_rng=False)


def _rewrite_state(path, mutate):
    """Replace ``state.pt`` by a mutated payload and re-sign it in the manifest, so only the content
    checks (not the checksum) can refuse it."""
    import hashlib
    payload = torch.load(path / "state.pt", weights_only=False)
    mutate(payload)
    torch.save(payload, path / "state.pt")
    data = (path / "state.pt").read_bytes()
    manifest = json.loads((path / "manifest.json").read_text())
    manifest["files"]["state.pt"] = {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data)}
    (path / "manifest.json").write_text(json.dumps(manifest))


def test_a_checksum_valid_nonfinite_payload_is_refused_without_mutation(tmp_path):
    _save(tmp_path / "ck", _model(1))
    name = next(iter(_model().state_dict()))
    _rewrite_state(tmp_path / "ck", lambda p: p["model"][name].view(-1)[0].fill_(float("nan")))
    target = _model(2)
    before = _clone_state(target)
    with pytest.raises((ValueError, FloatingPointError)):
        load_checkpoint(tmp_path / "ck", target, restore_rng=False)
    assert all(torch.equal(v, target.state_dict()[k]) for k, v in before.items())


@pytest.mark.parametrize("manifest", ["not json", "[]", '{"files": {}}',
                                      '{"files": {"state.pt": {"sha256": "xyz", "bytes": 1}}}'])
def test_a_malformed_manifest_is_refused_cleanly(tmp_path, manifest):
    _save(tmp_path / "ck", _model(1))
    (tmp_path / "ck" / "manifest.json").write_text(manifest)
    target = _model(2)
    before = _clone_state(target)
    with pytest.raises((ValueError, KeyError, TypeError)):
        load_checkpoint(tmp_path / "ck", target, restore_rng=False)
    assert all(torch.equal(v, target.state_dict()[k]) for k, v in before.items())


def test_a_second_publisher_never_replaces_a_checkpoint(tmp_path):
    first = _save(tmp_path / "ck", _model(1))
    with pytest.raises(FileExistsError):
        _save(tmp_path / "ck", _model(2))
    assert read_manifest(tmp_path / "ck")["files"] == first["files"]
    leftovers = [p.name for p in tmp_path.iterdir() if p.name != "ck"]
    assert leftovers == []  # the refused save's staging directory is gone


def test_a_composite_optimizer_mismatch_is_refused_before_the_model_changes(tmp_path):
    model = _model(1)
    muon = make_opt(model, TrainConfig(optimizer="muon", lr=0.02, aux_adamw_lr=0.003))
    _save(tmp_path / "ck", model, muon)
    target = _model(2)
    adamw = make_opt(target, TrainConfig(optimizer="adamw", lr=0.02))
    before = _clone_state(target)
    with pytest.raises((ValueError, KeyError, TypeError)):
        load_checkpoint(tmp_path / "ck", target, adamw, restore_rng=False)
    assert all(torch.equal(v, target.state_dict()[k]) for k, v in before.items())


def test_code_identity_covers_every_package_source(tmp_path):
    from pathlib import Path

    from tensor_train_ing_b200.checkpoint import code_identity
    ident = code_identity()
    text = json.dumps(ident)
    package = Path(__file__).resolve().parents[1] / "tensor_train_ing_b200"
    for nested in ("models/model.py", "ops/fused.py", "csrc/gemm/gemm.cu", "parallel/sharded.py"):
        if (package / nested).exists():
            assert Path(nested).name in text, nested
