"""Offline test helpers (package code never imports tests)."""
import torch


class FixtureTokenizer:
    """Character-code tokenizer with the GPT-2 end-of-text id; marked test-only in manifests."""
    name = "offline"
    eot_token = 50256

    def encode(self, text, **kwargs):
        return [ord(c) for c in text]


def state(path):
    return torch.load(path / "state.pt", weights_only=False, map_location="cpu")


# Smallest model shape used by the math and optimizer tests (vocab 97 padded to 128).
TINY_MODEL = dict(layers=2, d_model=32, heads=2, d_key=8, d_value=16, d_mlp=48, vocab_size=97, padded_vocab=128)
