"""Experiment configuration: ``ModelConfig``, ``TrainConfig`` and the YAML-backed ``Config``.

The field names, defaults and validation rules are the reference platform's public schema
(tnlm/config.py:15-138), so that its YAML files and the ``config`` blocks stored inside its
checkpoints load unchanged.  Unknown ``model``/``train`` keys are rejected; every other YAML
section (``project``, ``data``, ``evaluation``, ``b200`` ...) is kept verbatim in ``raw``.

Additions of this framework:
  * ``attention_backend`` also accepts ``"cuda"``; ``"triton"`` (the reference's name for its
    tiled kernel) selects the same hand-written sm_100a kernels here;
  * ``attention_backend="recurrent"`` runs polynomial attention in its chunked linear-state form
    (``models/long_context.py``): no T x T matrix, for very long contexts.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field, fields
from typing import Any

import yaml

MLP_KINDS = ("bilinear", "affine_bilinear", "swiglu")
ATTN_KINDS = ("signed_product", "offset_square", "lower_degree_mix", "softmax")
NORM_PACKAGES = ("pre_rms", "branch_rms", "sandwich_rms", "group_rms", "spectral_rms", "lagged", "taper")
FINAL_NORMS = ("rms", "lagged", "taper")
ATTN_BACKENDS = ("reference", "triton", "cuda", "auto", "recurrent")


@dataclass
class ModelConfig:
    layers: int = 12
    d_model: int = 512
    heads: int = 8
    d_key: int = 64
    d_value: int = 64
    d_mlp: int = 1664
    vocab_size: int = 50257
    padded_vocab: int = 50304
    tie_embeddings: bool = False
    mlp: str = "bilinear"
    attention: str = "signed_product"
    normalization: str = "pre_rms"
    final_normalization: str = "rms"
    rms_eps: float = 1.0e-6
    norm_groups: int = 4
    qk_norm: bool = False
    dropout: float = 0.0
    position_encoding: str = "rope"
    rope_base: float = 10000.0
    initialization: str = "explicit_fan_in_with_depth_scaled_outputs"
    residual_alpha: float = 1.0
    # std multiplier on the Q/K projections at init (1.0 = plain fan-in init)
    qk_init_scale: float = 1.0
    # polynomial attention row scale n_visible^-p; None = 0.5 (signed kinds) / 1.0 (offset_square)
    attn_row_power: float | None = None
    lagged_half_life_tokens: float = 1.0e6
    taper_ema_rate: float = 0.01
    offset_square_b: float = 1.0
    fp32_scores: bool = True
    # "reference" dense oracle; "cuda"/"triton" fused sm_100a kernels; "auto" = kernels on CUDA tensors
    attention_backend: str = "auto"
    activation_checkpointing: bool = False
    # chunked fused unembedding + cross-entropy when targets are given; 0 = dense logits
    loss_chunk_tokens: int = 0
    width_scaling_base: int | None = None
    width_lr_exponent: float = 0.5
    width_logit_exponent: float = 0.5
    depth_scaling_base: int | None = None
    depth_lr_exponent: float = 0.5
    depth_residual_base: int | None = None
    depth_residual_exponent: float = 1.0

    def __post_init__(self):
        _require(self.mlp in MLP_KINDS, f"mlp {self.mlp!r} not in {MLP_KINDS}")
        _require(self.attention in ATTN_KINDS, f"attention {self.attention!r} not in {ATTN_KINDS}")
        _require(self.normalization in NORM_PACKAGES, f"normalization {self.normalization!r}")
        _require(self.final_normalization in FINAL_NORMS, f"final_normalization {self.final_normalization!r}")
        _require(self.d_model % self.norm_groups == 0, "d_model must be divisible by norm_groups")
        _require(self.padded_vocab >= self.vocab_size, "padded_vocab must be >= vocab_size")
        _require(self.dropout == 0.0, "dropout is not part of this model family")
        _require(self.attention_backend in ATTN_BACKENDS, f"attention_backend {self.attention_backend!r}")
        _require(not (self.attention_backend == "recurrent" and self.attention == "softmax"),
                 "the recurrent attention backend is a polynomial-attention form (no softmax)")
        if self.normalization == "lagged" and self.final_normalization != "lagged":
            raise ValueError("lagged package requires final_normalization: lagged (else label it N)")
        if self.normalization == "taper" and self.final_normalization != "taper":
            raise ValueError("taper package requires final_normalization: taper "
                             "(else the final RMSNorm stays input-dependent)")
        stateful = {"taper", "lagged"} & {self.normalization, self.final_normalization}
        if self.activation_checkpointing and "taper" in stateful:
            raise ValueError("activation checkpointing would double-count TaperNorm statistics and anchor terms")
        if self.activation_checkpointing and "lagged" in stateful:
            raise ValueError("activation checkpointing would double-count lagged statistics")
        if self.qk_norm:
            raise NotImplementedError("qk_norm needs head scope/eps/gain/RoPE order spec")


@dataclass
class TrainConfig:
    optimizer: str = "adamw"
    lr: float = 4.5e-4
    beta1: float = 0.9
    beta2: float = 0.9872585449
    weight_decay_hidden: float = 0.1
    grad_clip: float = 1.0
    global_prediction_tokens_per_update: int = 8192
    rung_total_tokens: int = 100_000_000
    schedule: str = "constant_with_separate_cooldown"
    cooldown_fraction: float = 0.1
    bf16_compute: bool = True
    fp32_norm_reductions: bool = True
    fp32_optimizer_state: bool = True
    compile: bool = True
    seed: int = 101
    deterministic: bool = False
    stability_every_steps: int = 0
    taper_anchor_lambda: float = 0.1
    taper_end_fraction: float = 1.0
    qk_clip_tau: float = 0.0
    qk_clip_every_steps: int = 0
    qk_clip_source: str = "probe"
    muon_momentum: float = 0.95
    muon_adjust_lr: str = "match_rms_adamw"
    aux_adamw_lr: float | None = None


def _require(cond: bool, msg: str):
    if not cond:
        raise AssertionError(msg)


def _from_section(cls, section: dict[str, Any] | None):
    if section is not None and not isinstance(section, dict):
        raise ValueError(f"the {cls.__name__} section must be a mapping, not {type(section).__name__}")
    values = dict(section or {})
    known = {f.name for f in fields(cls)}
    extra = sorted(set(values) - known)
    if extra:
        raise ValueError(f"unknown {cls.__name__} keys: {extra}")
    return cls(**values)


@dataclass
class Config:
    model: ModelConfig = field(default_factory=ModelConfig)
    train: TrainConfig = field(default_factory=TrainConfig)
    raw: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, raw: dict) -> "Config":
        if raw is not None and not isinstance(raw, dict):
            # e.g. a sweep candidate list: dict() would read each two-key entry as a key/value pair
            raise ValueError(f"a configuration must be a mapping of sections, not {type(raw).__name__}")
        raw = dict(raw or {})
        return cls(model=_from_section(ModelConfig, raw.get("model")),
                   train=_from_section(TrainConfig, raw.get("train")), raw=raw)

    @classmethod
    def from_yaml(cls, path: str) -> "Config":
        with open(path) as fh:
            return cls.from_dict(yaml.safe_load(fh) or {})

    def to_dict(self) -> dict:
        """Every raw section plus the resolved ``model`` and ``train`` blocks."""
        out = dict(self.raw)
        out["model"] = asdict(self.model)
        out["train"] = asdict(self.train)
        return out
