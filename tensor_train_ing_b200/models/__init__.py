"""Model family: TensorLM (bilinear MLP + polynomial attention) and the SwiGLU/softmax control."""
from .model import MLP, PACKAGES, Attention, Block, TensorLM, linear_weight, score_bound  # noqa: F401
