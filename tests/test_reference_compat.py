"""Checkpoint and numerics compatibility with the reference package (installed offline under
baseline/_ref; skipped where it is absent): state dicts load both ways and give the same logits."""
import os
import sys

import pytest
import torch

from helpers import TINY_MODEL

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def tnlm():
    if not os.path.isdir(os.path.join(REF, "tnlm")):
        pytest.skip("reference package not installed")
    sys.path.insert(0, REF)
    try:
        import tnlm.checkpoint
        import tnlm.config
        import tnlm.model
        import tnlm.optim
        yield tnlm
    finally:
        sys.path.remove(REF)


@pytest.mark.parametrize("normalization", ["pre_rms", "group_rms", "sandwich_rms", "spectral_rms"])
@pytest.mark.parametrize("attention", ["signed_product", "offset_square", "lower_degree_mix"])
def test_reference_checkpoint_loads_with_identical_logits(tnlm, tmp_path, normalization, attention):
    from tensor_train_ing_b200.checkpoint import load_checkpoint
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    kw = dict(TINY_MODEL, normalization=normalization, attention=attention)
    torch.manual_seed(3)
    ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**kw)).double().eval()
    tnlm.checkpoint.save_checkpoint(tmp_path / "ck", ref, None, None, config={"model": kw}, progress={"steps": 0},
                                    manifest_hash="0" * 64)
    ours = TensorLM(ModelConfig(**kw)).double().eval()
    load_checkpoint(tmp_path / "ck", ours, restore_rng=False)
    idx = torch.randint(0, 97, (2, 11))
    doc = torch.tensor([[0] * 6 + [1] * 5, [0] * 11])
    with torch.no_grad():
        a = ref(idx, doc_ids=doc)
        b = ours(idx, doc_ids=doc)
    torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-10)


def test_our_checkpoint_loads_in_reference(tnlm, tmp_path):
    from tensor_train_ing_b200.checkpoint import save_checkpoint
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    torch.manual_seed(4)
    ours = TensorLM(ModelConfig(**TINY_MODEL)).eval()
    save_checkpoint(tmp_path / "ck", ours, None, None, config={"model": TINY_MODEL}, progress={"steps": 0},
                    manifest_hash="0" * 64)
    ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**TINY_MODEL)).eval()
    tnlm.checkpoint.load_checkpoint(tmp_path / "ck", ref, restore_rng=False)
    idx = torch.randint(0, 97, (1, 9))
    with torch.no_grad():
        torch.testing.assert_close(ref(idx), ours(idx))


def test_same_seed_same_initialisation(tnlm):
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    torch.manual_seed(11)
    ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**TINY_MODEL))
    torch.manual_seed(11)
    ours = TensorLM(ModelConfig(**TINY_MODEL))
    rs, os_ = ref.state_dict(), ours.state_dict()
    assert rs.keys() == os_.keys()
    for k in rs:
        assert torch.equal(rs[k], os_[k]), k
