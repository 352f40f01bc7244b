"""The streamed, component-at-a-time initialisation is the serial ``TensorLM(cfg)`` initialisation,
bit for bit, and leaves the CPU generator where serial construction leaves it."""
import pytest
import torch

from tensor_train_ing_b200.config import ModelConfig
from tensor_train_ing_b200.models.init_stream import named_device_initial_tensors, named_initial_tensors
from tensor_train_ing_b200.models.model import TensorLM


@pytest.mark.parametrize("norm", ["pre_rms", "spectral_rms", "lagged", "taper", "sandwich_rms"])
@pytest.mark.parametrize("tie", [False, True])
def test_streamed_initialisation_is_serial(norm, tie):
    extra = {"final_normalization": norm} if norm in ("lagged", "taper") else {}
    cfg = ModelConfig(vocab_size=500, padded_vocab=512, d_model=64, layers=3, heads=2, d_key=32, d_value=32,
                      d_mlp=128, normalization=norm, tie_embeddings=tie, **extra)
    torch.manual_seed(5)
    serial = TensorLM(cfg).state_dict()
    after_serial = torch.get_rng_state()
    torch.manual_seed(5)
    streamed = dict(named_initial_tensors(cfg))
    assert torch.equal(torch.get_rng_state(), after_serial)
    if tie:
        streamed["unembed.weight"] = streamed["embed.weight"]
    assert set(serial) <= set(streamed)  # (the stream also carries non-persistent buffers)
    for k, v in serial.items():
        assert torch.equal(v, streamed[k]), k


def test_device_initialisation_has_every_tensor():
    cfg = ModelConfig(vocab_size=500, padded_vocab=512, d_model=64, layers=2, heads=2, d_key=32, d_value=32,
                      d_mlp=128)
    torch.manual_seed(0)
    names = dict(named_device_initial_tensors(cfg, "cpu"))
    assert set(TensorLM(cfg).state_dict()) <= set(names)
    assert abs(float(names["embed.weight"].std()) - 1.0) < 0.05
