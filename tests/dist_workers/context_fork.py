"""Worker: a distributed run forked to a longer context on gloo ranks.

A two-step parent at context 8 is resumed at context 16 with ``context_fork=True``: the fork is
recorded in the context history, the token count continues from the parent's, a plain resume at the
new context is refused, and two forks of the same parent give the same losses and weights.  Prints
``FORK_OK`` on rank 0.  argv: <shared tmp dir>."""
import copy
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "dist_workers"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from train_replay import config  # noqa: E402
from helpers import FixtureTokenizer  # noqa: E402
from tensor_train_ing_b200.data import prepare_data  # noqa: E402
from tensor_train_ing_b200.distributed_train import distributed_train_run  # noqa: E402


def main():
    tmp = Path(sys.argv[1])
    os.environ["TTB_SHARD_PARAMS"] = "0"
    dist.init_process_group("gloo")
    rank = dist.get_rank()
    torch.set_num_threads(1)
    if rank == 0:
        src = tmp / "source.jsonl"
        src.write_text("".join(json.dumps({"id": str(i), "text": "abcdefghijklm" * (1 + i % 3)}) + "\n"
                               for i in range(30)))
        prepare_data(tmp / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                     split_fractions={"train": .8, "val": 0., "test": 0., "calibration": .2})
    dist.barrier()
    cfg = config(tmp)
    parent = distributed_train_run(cfg, tmp / "parent", max_steps=2, max_seconds=300, device="cpu")
    longer = copy.deepcopy(cfg)
    longer.raw["data"]["context"] = 16
    refused = False
    try:
        distributed_train_run(longer, tmp / "plain", max_steps=1, max_seconds=300, device="cpu",
                              resume=parent["checkpoint"])
    except ValueError:
        refused = True
    assert refused, "a context change must need the explicit fork"
    runs = []
    for name in ("fork_a", "fork_b"):
        out = distributed_train_run(longer, tmp / name, max_steps=2, max_seconds=300, device="cpu",
                                    resume=parent["checkpoint"], context_fork=True, export_max_state_bytes=10 ** 9)
        runs.append(out)
    hist = runs[0]["progress"]["context_history"]
    assert [h["context"] for h in hist] == [8, 16], hist
    assert runs[0]["progress"]["steps"] == 4
    assert runs[0]["progress"]["tokens"] == parent["progress"]["tokens"] + 2 * 12
    if rank == 0:
        losses = [[json.loads(x)["loss"] for x in (tmp / n / "metrics.jsonl").read_text().splitlines()]
                  for n in ("fork_a", "fork_b")]
        assert losses[0] == losses[1], losses
        a = torch.load(tmp / "fork_a" / "final-weights" / "state.pt", weights_only=False)["model"]
        b = torch.load(tmp / "fork_b" / "final-weights" / "state.pt", weights_only=False)["model"]
        assert all(torch.equal(a[k], b[k]) for k in a)
        print("FORK_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
