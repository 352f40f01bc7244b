"""Worker: sharded checkpoints move between the reference's distributed trainer and this one.

argv: <shared tmp dir> <adamw|muon>.  On two gloo ranks: the reference trains two updates and saves
``tnlm-dcp-v1``; both trainers resume it for two more updates.  Then this trainer trains two
updates saving ``tnlm-dcp-v1``; both resume that.  Rank 0 writes every run's losses to
``losses.json`` and prints ``DCP_INTERCHANGE_OK``."""
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))

import tnlm.config  # noqa: E402
import tnlm.distributed_train  # noqa: E402
import yaml  # noqa: E402
from helpers import FixtureTokenizer  # noqa: E402
from tensor_train_ing_b200.config import Config  # noqa: E402
from tensor_train_ing_b200.data import prepare_data  # noqa: E402
from tensor_train_ing_b200.distributed_train import distributed_train_run  # noqa: E402


def losses(run_dir: Path) -> list:
    return [json.loads(x)["loss"] for x in (run_dir / "metrics.jsonl").read_text().splitlines()]


def main():
    tmp, optimizer = Path(sys.argv[1]), sys.argv[2]
    os.environ["TTB_SHARD_PARAMS"] = "0"
    dist.init_process_group("gloo")
    rank = dist.get_rank()
    torch.set_num_threads(1)
    if rank == 0 and not (tmp / "data").exists():
        src = tmp / "source.jsonl"
        src.write_text("".join(json.dumps({"id": str(i), "text": "abcdefghijklm" * (1 + i % 3)}) + "\n"
                               for i in range(30)))
        prepare_data(tmp / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                     split_fractions={"train": .8, "val": 0., "test": 0., "calibration": .2})
        doc = {"model": {"layers": 1, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                         "padded_vocab": 50257},
               "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 12,
                         "rung_total_tokens": 200, "lr": 0.01, "optimizer": optimizer},
               "data": {"manifest": str(tmp / "data" / "manifest.json"), "context": 8, "micro_batch_size": 1},
               "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp / "spend.json")}}
        (tmp / "run.yaml").write_text(yaml.safe_dump(doc))
    dist.barrier()
    ours = lambda: Config.from_yaml(str(tmp / "run.yaml"))  # noqa: E731
    theirs = lambda: tnlm.config.Config.from_yaml(str(tmp / "run.yaml"))  # noqa: E731
    run = {"max_steps": 2, "max_seconds": 300, "device": "cpu"}
    # reference -> here
    a = tnlm.distributed_train.distributed_train_run(theirs(), tmp / "ref-a", **run)
    tnlm.distributed_train.distributed_train_run(theirs(), tmp / "ref-b", resume=a["checkpoint"], **run)
    distributed_train_run(ours(), tmp / "ours-b", resume=a["checkpoint"], **run)
    # here -> reference
    c = distributed_train_run(ours(), tmp / "ours-c", checkpoint_format="tnlm-dcp-v1", **run)
    distributed_train_run(ours(), tmp / "ours-d", resume=c["checkpoint"], **run)
    tnlm.distributed_train.distributed_train_run(theirs(), tmp / "ref-d", resume=c["checkpoint"], **run)
    if rank == 0:
        names = ("ref-a", "ref-b", "ours-b", "ours-c", "ours-d", "ref-d")
        (tmp / "losses.json").write_text(json.dumps({n: losses(tmp / n) for n in names}))
        print("DCP_INTERCHANGE_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
