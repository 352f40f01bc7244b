"""Worker: distributed trainer on gloo.  Checks that a resumed run replays an uninterrupted one
bitwise and writes the final parameters for comparison with the serial trainer.

argv: <shared tmp dir> [mode].  Modes: replicated, shard (the fp32 parameters are sharded over the
ranks, owners only, and the comparisons use the exported full weights), lagged, taper, cosine (the
fixed-horizon schedule), muon (Muon on the hidden matrices) and qkclip (QK-clip every update from
the batch score bounds, with a threshold every head exceeds; qkclip-shard the same with sharded
parameters, where only owners rescale and the gather brings the result).  Prints ``REPLAY_OK`` on
rank 0."""
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from helpers import FixtureTokenizer  # noqa: E402
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig  # noqa: E402
from tensor_train_ing_b200.data import prepare_data  # noqa: E402
from tensor_train_ing_b200.distributed_train import distributed_train_run  # noqa: E402


def config(tmp, mode="replicated"):
    model = dict(layers=1, d_model=8, heads=1, d_key=4, d_value=4, d_mlp=12, padded_vocab=50257)
    if mode in ("lagged", "taper"):
        model.update(normalization=mode, final_normalization=mode)
    cfg = Config(model=ModelConfig(**model),
                 train=TrainConfig(compile=False, bf16_compute=False, global_prediction_tokens_per_update=12,
                                   rung_total_tokens=200, lr=.01),
                 raw={"data": {"manifest": str(tmp / "data" / "manifest.json"), "context": 8, "micro_batch_size": 1,
                               "calibration_tokens": 16},
                      "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp / "spend.json")}})
    if mode in ("taper", "cosine"):
        cfg.train.rung_total_tokens = 12 * 300  # the gate / the decay must end after the 100-update warm-up
    if mode == "cosine":
        cfg.train.schedule = "cosine"
    if mode == "muon":
        cfg.train.optimizer = "muon"
        cfg.train.aux_adamw_lr = .01
    if mode.startswith("qkclip"):
        cfg.train.qk_clip_tau = 1e-3
        cfg.train.qk_clip_every_steps = 1
        cfg.train.qk_clip_source = "batch_bound"
    return cfg


def main():
    tmp = Path(sys.argv[1])
    mode = sys.argv[2] if len(sys.argv) > 2 else "replicated"
    shard = mode in ("shard", "qkclip-shard")
    os.environ["TTB_SHARD_PARAMS"] = "1" if shard else "0"
    dist.init_process_group("gloo")
    rank = dist.get_rank()
    torch.set_num_threads(1)
    if rank == 0 and not (tmp / "data").exists():
        src = tmp / "source.jsonl"
        src.write_text("".join(json.dumps({"id": str(i), "text": "abcdefghijklm" * (1 + i % 3)}) + "\n"
                               for i in range(30)))
        prepare_data(tmp / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                     split_fractions={"train": .8, "val": 0., "test": 0., "calibration": .2})
    dist.barrier()
    cfg = config(tmp, mode)
    export = 10 ** 9
    full = distributed_train_run(cfg, tmp / "full", max_steps=4, max_seconds=300, device="cpu",
                                 export_max_state_bytes=export)
    first = distributed_train_run(cfg, tmp / "a", max_steps=2, max_seconds=300, device="cpu")
    second = distributed_train_run(cfg, tmp / "b", max_steps=2, max_seconds=300, device="cpu", resume=first["checkpoint"],
                                   export_max_state_bytes=export)
    assert full["progress"]["steps"] == second["progress"]["steps"] == 4
    assert full["progress"]["tokens"] == second["progress"]["tokens"] == 48
    if rank == 0:
        a = torch.load(tmp / "full" / "final-weights" / "state.pt", weights_only=False)["model"]
        b = torch.load(tmp / "b" / "final-weights" / "state.pt", weights_only=False)["model"]
        for k in a:
            assert torch.equal(a[k], b[k]), k
        if shard:  # the recovery checkpoint's model.pt holds only what every rank replicates
            m = torch.load(tmp / "full" / "final" / "model.pt", weights_only=False)["model"]
            assert "blocks.0.mlp.l.weight" not in m and "embed.weight" in m
        losses = [json.loads(x)["loss"] for x in (tmp / "full" / "metrics.jsonl").read_text().splitlines()]
        (tmp / "distributed_losses.json").write_text(json.dumps(losses))
        print("REPLAY_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
