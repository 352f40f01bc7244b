"""tensor_train_ing_b200: a B200-native training framework for tensor-network language models
(bilinear MLP + polynomial attention), with the public surface of the reference ``tnlm``
platform: ``Config``, ``TensorLM``, ``make_optimizer``, trainers, checkpoints and the CLI."""
from .config import Config, ModelConfig, TrainConfig  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    if name == "TensorLM":
        from .models.model import TensorLM
        return TensorLM
    raise AttributeError(name)
