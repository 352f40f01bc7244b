"""Model-shape presets, parameter counts and a capacity planner for this framework's memory layout
(reference tnlm/shapes.py:23-110).

Presets: the reference's named shapes (same names, layer counts, widths, heads and head dims, and
its parameter-matched polynomial MLP width d_mlp_poly = round((d_mlp_softmax - 2d/3) / 128) * 128,
with the reference's exact small-model widths), plus the shapes this framework benchmarks
(``bench_1b``, ``bench_7b``, ``bench_32b``: bilinear MLP at 4x width as in the benchmark
configs).  Parameter counts instantiate a block on the meta device (never formulas).

Capacity model (per GPU, owner-computes sharded data parallelism over ``gpus`` ranks):

* replicated: fp32 parameters (4 B), fp32 gradient accumulation buffer (4 B) and the bf16 operand
  caches of the fused GEMMs (2 B) for every parameter;
* sharded: optimizer state of the owned parameters, Muon momentum (4 B) for hidden matrices and
  two AdamW moments (8 B) for the rest;
* activations of one micro-batch saved for backward by the fused block, counted from what
  ``ops/block.py`` keeps per token and layer: the fp32 residual stream (4d), bf16 normed inputs of
  both branches (2 * 2d), the bf16 q1|k1|q2|k2|v buffer (2 * 5 * H * dk for the signed product),
  the bf16 attention output (2 * H * dv), the bf16 bilinear factors l and r (2 * 2 * d_mlp) and the
  per-row norm statistics; with activation checkpointing only the block inputs (4d) stay, plus one
  block's full set during its recompute;
* the loss workspace: one chunk of fp32 logit partials (the fused CE never stores logits) and the
  backward's bf16 dlogits chunk.

It is a capacity plan, not a fit proof: compare with ``torch.cuda.max_memory_allocated`` of a run.
"""
from __future__ import annotations

import torch

from ..config import ModelConfig

# name: (layers, d_model, heads, head_dim, d_mlp_softmax)
_BASE = {
    "screen_100m": (12, 512, 8, 64, 2048),
    "confirm_500m": (24, 1024, 16, 64, 4096),
    "width_1024_12l": (12, 1024, 16, 64, 4096),
    "pilot_1b": (24, 2048, 16, 128, 5504),
    "pilot_3b": (32, 2560, 20, 128, 6912),
    "funded_7b": (32, 4096, 32, 128, 11008),
    "funded_32b": (64, 5120, 40, 128, 27648),
}
_EXACT_POLY_MLP = {"screen_100m": 1664, "confirm_500m": 3392, "width_1024_12l": 3392}
# benchmark shapes: (layers, d_model, heads, head_dim, bilinear d_mlp)
_BENCH = {
    "bench_100m": (12, 768, 12, 64, 3072),
    "bench_1b": (24, 2048, 16, 128, 8192),
    "bench_7b": (32, 4096, 32, 128, 16384),
    "bench_32b": (48, 6144, 48, 128, 24576),
}


def preset(name: str, polynomial: bool = True, **overrides) -> ModelConfig:
    if name in _BENCH:
        L, d, H, hd, m = _BENCH[name]
        kw = dict(attention="signed_product", mlp="bilinear", d_mlp=m) if polynomial else \
            dict(attention="softmax", mlp="swiglu", d_mlp=m)
    else:
        L, d, H, hd, m_soft = _BASE[name]
        if polynomial:
            m = _EXACT_POLY_MLP.get(name) or int(round((m_soft - 2 * d / 3) / 128) * 128)
            kw = dict(attention="signed_product", mlp="bilinear", d_mlp=m)
        else:
            kw = dict(attention="softmax", mlp="swiglu", d_mlp=m_soft)
    kw.update(layers=L, d_model=d, heads=H, d_key=hd, d_value=hd)
    kw.update(overrides)
    return ModelConfig(**kw)


def preset_names() -> list[str]:
    return list(_BASE) + list(_BENCH)


def count_params(cfg: ModelConfig) -> dict:
    from .model import Block
    with torch.device("meta"):
        blk = Block(cfg)
    per_block = sum(p.numel() for p in blk.parameters())
    per_block_mat = sum(p.numel() for p in blk.parameters() if p.dim() >= 2)
    emb = cfg.padded_vocab * cfg.d_model * (1 if cfg.tie_embeddings else 2)
    return {"total": cfg.layers * per_block + emb + cfg.d_model, "matrices": cfg.layers * per_block_mat + emb,
            "non_embedding": cfg.layers * per_block_mat, "per_block": per_block, "embedding": emb}


def activation_bytes_per_token_layer(cfg: ModelConfig) -> float:
    d, H = cfg.d_model, cfg.heads
    qk = 4 if cfg.attention in ("signed_product", "lower_degree_mix") else 2
    qkv = 2 * (qk * H * cfg.d_key + H * cfg.d_value)
    return 4 * d + 2 * 2 * d + qkv + 2 * H * cfg.d_value + 2 * 2 * cfg.d_mlp + 16


def largest_weight_group(cfg: ModelConfig) -> int:
    """Elements of the largest matrix group one GEMM reads (fused QKV, one bilinear factor, the down
    projection or the unembedding): the size of a gather staging slot."""
    d, H = cfg.d_model, cfg.heads
    qk = 4 if cfg.attention in ("signed_product", "lower_degree_mix") else 2
    qkv = (qk * H * cfg.d_key + H * cfg.d_value) * d
    return max(qkv, cfg.d_mlp * d, cfg.padded_vocab * d)


def memory_plan(cfg: ModelConfig, *, gpus: int, micro_tokens_per_gpu: int, gpu_gb: float = 180.0,
                checkpointing: bool | None = None, workspace_gb: float = 4.0, optimizer: str = "muon",
                shard_params: bool = False, fused_gather: bool = True, gather_slots: int = 8,
                kept_blocks: int = 0) -> dict:
    """Per-GPU bytes of the owner-computes layout plus one micro-batch of activations.

    Replicated layout: fp32 parameters and gradients and the bf16 GEMM caches on every rank, the
    optimizer state sharded.  ``shard_params``: the block matrices and the unembedding keep fp32
    master, gradient accumulator and optimizer state only on their owner (1/gpus each) and two
    per-block fp32 staging slots; their bf16 rows are split across the ranks (1/gpus each) and
    gathered by the consuming GEMMs into ``gather_slots`` staging slots (``fused_gather``), or held
    in full on every rank; embedding and vectors replicated.  ``kept_blocks``: under checkpointing,
    blocks whose activations are kept rather than recomputed (the engine's ``recompute_blocks`` is
    the layer count minus this)."""
    ckpt = cfg.activation_checkpointing if checkpointing is None else checkpointing
    c = count_params(cfg)
    n = c["total"]
    hidden = c["non_embedding"]
    unembed = 0 if cfg.tie_embeddings else cfg.padded_vocab * cfg.d_model
    if optimizer == "muon":
        opt = (4 * hidden + 8 * (n - hidden)) / gpus
    else:
        opt = 8 * n / gpus
    if shard_params:
        sharded = hidden + unembed
        staging = 2 * 4 * max(c["per_block"], unembed)
        bf16 = 2 * sharded / gpus + 2 * gather_slots * largest_weight_group(cfg) if fused_gather else 2 * sharded
        weights = bf16 + 8 * sharded / gpus + 10 * (n - sharded) + staging
    else:
        weights = (4 + 4 + 2) * n
    per_layer = activation_bytes_per_token_layer(cfg)
    if ckpt:
        act = (4 * cfg.d_model * cfg.layers + per_layer * (1 + min(kept_blocks, cfg.layers))) * micro_tokens_per_gpu
    else:
        act = per_layer * cfg.layers * micro_tokens_per_gpu
    chunk = min(micro_tokens_per_gpu, cfg.loss_chunk_tokens or micro_tokens_per_gpu)
    loss = 2 * chunk * cfg.padded_vocab + 8 * micro_tokens_per_gpu
    total = weights + opt + act + loss + workspace_gb * 1e9
    layout = ("owner-computes, parameter-sharded: fp32 masters/grads/optimizer state on owners, bf16 rows "
              + ("split across ranks and gathered by the GEMMs" if fused_gather else "replicated")
              if shard_params else
              "owner-computes: replicated fp32 params/grads + bf16 caches, sharded optimizer state")
    return {"params_B": round(n / 1e9, 3), "gpus": gpus, "micro_tokens_per_gpu": micro_tokens_per_gpu,
            "checkpointing": ckpt, "shard_params": shard_params, "replicated_state_GB": round(weights / 1e9, 1),
            "optimizer_state_GB": round(opt / 1e9, 1), "activations_GB": round(act / 1e9, 1),
            "loss_GB": round(loss / 1e9, 2), "total_GB": round(total / 1e9, 1), "fits": total < 0.92 * gpu_gb * 1e9,
            "layout": layout}


def blocks_to_recompute(cfg: ModelConfig, *, gpus: int, micro_tokens_per_gpu: int, device_bytes: float,
                        shard_params: bool = False, fill: float = 0.92, optimizer: str = "muon") -> int:
    """Selective recompute: how many of the first blocks to recompute under activation checkpointing so
    that the plan with the other blocks' activations kept stays within ``fill`` of the device (all
    of them when nothing more fits; never fewer than zero)."""
    plan = memory_plan(cfg, gpus=gpus, micro_tokens_per_gpu=micro_tokens_per_gpu, gpu_gb=device_bytes / 1e9,
                       checkpointing=True, shard_params=shard_params, optimizer=optimizer)
    room = fill * device_bytes - plan["total_GB"] * 1e9
    per_block = activation_bytes_per_token_layer(cfg) * micro_tokens_per_gpu
    kept = max(0, min(cfg.layers, int(room // per_block)))
    return cfg.layers - kept


def needs_parameter_sharding(cfg: ModelConfig, world: int, device=None) -> bool:
    """Whether a data-parallel engine should shard the fp32 parameters: ``TTB_SHARD_PARAMS=1``/``0``
    decides; otherwise yes when the replicated fp32 parameters, gradients and bf16 caches would
    take more than 60% of the device's memory and there is more than one rank."""
    import os
    env = os.environ.get("TTB_SHARD_PARAMS")
    if env is not None:
        return env not in ("0", "")
    if world <= 1:
        return False
    total = 180e9
    if device is not None and torch.device(device).type == "cuda" and torch.cuda.is_available():
        total = torch.cuda.get_device_properties(torch.device(device)).total_memory
    return 10 * count_params(cfg)["total"] > 0.6 * total


def min_gpus(cfg: ModelConfig, micro_tokens_per_gpu: int, gpu_gb: float = 180.0, checkpointing: bool = True,
             max_gpus: int = 1024) -> dict | None:
    """Smallest power-of-two GPU count whose plan fits: the replicated layout first, then the
    parameter-sharded one."""
    g = 1
    while g <= max_gpus:
        for shard in (False, True) if g > 1 else (False,):
            plan = memory_plan(cfg, gpus=g, micro_tokens_per_gpu=micro_tokens_per_gpu, gpu_gb=gpu_gb,
                               checkpointing=checkpointing, shard_params=shard)
            if plan["fits"]:
                return plan
        g *= 2
    return None


def table(micro_tokens_per_gpu: int = 8192, gpu_gb: float = 180.0) -> list[dict]:
    rows = []
    for name in preset_names():
        for poly in (True, False):
            cfg = preset(name, poly, loss_chunk_tokens=8192)
            c = count_params(cfg)
            plan = min_gpus(cfg, micro_tokens_per_gpu, gpu_gb)
            rows.append({"preset": name, "family": "polynomial" if poly else "softmax-control",
                         "layers": cfg.layers, "d_model": cfg.d_model, "heads": cfg.heads, "head_dim": cfg.d_key,
                         "d_mlp": cfg.d_mlp, "params_B": round(c["matrices"] / 1e9, 3),
                         "min_gpus_ckpt": plan["gpus"] if plan else None,
                         "per_gpu_GB": plan["total_GB"] if plan else None})
    return rows


if __name__ == "__main__":
    import json
    for r in table():
        print(json.dumps(r))
