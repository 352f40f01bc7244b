"""Fixtures shared by the CPU and GPU tests.  Nothing in the package imports this module."""
import torch


class FixtureTokenizer:
    """Maps each character to its code point and ends documents with id 50256 (GPT-2's end of
    text), so fixture datasets need no vocabulary files; manifests built with it are flagged
    ``test_only`` and the trainers refuse them on a GPU."""
    name = "offline"
    eot_token = 50256

    def encode(self, text, **kwargs):
        return list(map(ord, text))


def state(path):
    """The unpickled ``state.pt`` payload of the checkpoint directory ``path``."""
    return torch.load(path / "state.pt", weights_only=False, map_location="cpu")


# Two layers of width 32: the model shape of the numerics and optimizer unit tests.  A vocabulary
# of 97 real ids padded to 128 exercises the padded-logit masking.
TINY_MODEL = {"layers": 2, "d_model": 32, "heads": 2, "d_key": 8, "d_value": 16, "d_mlp": 48, "vocab_size": 97,
              "padded_vocab": 128}
