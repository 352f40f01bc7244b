"""The serial initialisation of ``TensorLM`` streamed one top-level component at a time.

A parameter-sharded run never materialises the whole fp32 model on one rank, yet its weights must
be the ones ``TensorLM(cfg)`` would draw on the CPU under the same seed (the reference gives the same
guarantee, tnlm/initialization.py canonical_initialization_components and
tnlm/sharded_initialization.py:38-61).  Serial construction consumes the CPU generator in two
phases: the module constructors (embed, blocks 0..L-1, final norm, unembed, each drawing its own
default init) and then ``reset_parameters`` (embed, blocks, unembed).  So:

  pass 1  construct each component on the CPU and drop it, recording the generator state before
          each constructor; the state after the last one is where the reset phase starts;
  pass 2  for each component, rebuild it from its recorded constructor state, then run its reset
          draws from the running reset-phase state, and hand it to the caller.

Only one component (a block, or a vocabulary matrix) exists at a time.  When the iterator is
exhausted the CPU generator is exactly where ``TensorLM(cfg)`` leaves it.
"""
from __future__ import annotations

from typing import Callable, Iterator

import torch
import torch.nn as nn

from ..config import ModelConfig
from .model import Block, init_block, init_embedding, init_unembedding
from .normalization import make_norm


def _components(cfg: ModelConfig) -> list[tuple[str, Callable[[], nn.Module], Callable | None]]:
    """(state-dict prefix, constructor, reset draws) in TensorLM's construction order."""
    out = [("embed", lambda: nn.Embedding(cfg.padded_vocab, cfg.d_model), init_embedding)]
    out += [(f"blocks.{i}", lambda: Block(cfg), lambda m: init_block(m, cfg)) for i in range(cfg.layers)]
    out.append(("final_norm", lambda: make_norm(cfg.final_normalization, cfg.d_model, cfg), None))
    out.append(("unembed", lambda: nn.Linear(cfg.d_model, cfg.padded_vocab, bias=False),
                None if cfg.tie_embeddings else init_unembedding))
    return out


def stream_initialization(cfg: ModelConfig) -> Iterator[tuple[str, nn.Module]]:
    """Yield (prefix, CPU module) with the values serial construction gives each component.

    The caller seeds the CPU generator first (as for ``TensorLM(cfg)``) and must drop each module
    before advancing.  With tied embeddings the unembedding is not yielded (it is ``embed``)."""
    comps = _components(cfg)
    starts = []
    with torch.device("cpu"):
        for _, make, _ in comps:
            starts.append(torch.get_rng_state())
            make()
    reset_state = torch.get_rng_state()
    try:
        for (prefix, make, init), start in zip(comps, starts):
            if prefix == "unembed" and cfg.tie_embeddings:
                continue
            torch.set_rng_state(start)
            with torch.device("cpu"):
                module = make()
            torch.set_rng_state(reset_state)
            if init is not None:
                init(module)
            reset_state = torch.get_rng_state()
            yield prefix, module
            del module
    finally:
        torch.set_rng_state(reset_state)


def named_initial_tensors(cfg: ModelConfig) -> Iterator[tuple[str, torch.Tensor]]:
    """Every parameter and buffer of the serial initialisation as (state-dict name, CPU tensor),
    component by component."""
    for prefix, module in stream_initialization(cfg):
        for name, t in list(module.named_parameters()) + list(module.named_buffers()):
            yield f"{prefix}.{name}", t.detach()
        del module


def named_device_initial_tensors(cfg: ModelConfig, device) -> Iterator[tuple[str, torch.Tensor]]:
    """The same per-component distributions drawn on ``device`` with its own generator (seed it
    first): every rank that draws with the same seed gets the same values, in a fraction of the
    serial CPU time, but not the serial initialisation's values.  For throughput runs of models
    whose serial CPU initialisation would take minutes."""
    for prefix, make, init in _components(cfg):
        if prefix == "unembed" and cfg.tie_embeddings:
            continue
        with torch.device(device):
            module = make()
        if init is not None:
            init(module)
        for name, t in list(module.named_parameters()) + list(module.named_buffers()):
            yield f"{prefix}.{name}", t.detach()
        del module
