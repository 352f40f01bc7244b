"""Worker: host-side failure injection on gloo ranks.

argv: <scenario> <tmp dir>.  Scenarios:
  phase        rank 1 raises inside a _phase callback -> every rank raises the same ValueError
  corrupt      a rank file of a sharded checkpoint is corrupted -> load fails on every rank, nothing installed
  dead_rank    rank 1 leaves before a collective -> rank 0's collective ends with an error (short timeout)
  nonfinite    one rank's gradient holds an inf -> the update refuses on every rank, weights untouched
  disk_full    the filesystem reports no space to rank 0 -> the sharded save fails on every rank and
               leaves no directory behind
Prints ``SCENARIO_OK <scenario>`` from every rank that observed the expected failure."""
import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from tensor_train_ing_b200.config import ModelConfig, TrainConfig  # noqa: E402
from tensor_train_ing_b200.distributed_checkpoint import (_phase, load_distributed_checkpoint,  # noqa: E402
                                                          save_distributed_checkpoint)
from tensor_train_ing_b200.models.model import TensorLM  # noqa: E402
from tensor_train_ing_b200.optim import make_optimizer  # noqa: E402
from tensor_train_ing_b200.parallel.sharded import ShardedDataParallel  # noqa: E402


def main():
    scenario, tmp = sys.argv[1], Path(sys.argv[2])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=10))
    rank = dist.get_rank()
    if scenario == "phase":
        def work():
            if rank == 1:
                raise RuntimeError("injected rank-1 failure")
            return 7
        try:
            _phase("injected", work)
        except ValueError as e:
            assert "rank 1: RuntimeError: injected rank-1 failure" in str(e), str(e)
            print(f"SCENARIO_OK {scenario}", flush=True)
    elif scenario == "corrupt":
        torch.manual_seed(0)
        cfg = ModelConfig(layers=1, d_model=16, heads=2, d_key=4, d_value=4, d_mlp=8, vocab_size=31, padded_vocab=32)
        model = TensorLM(cfg)
        dp = ShardedDataParallel(model, "cpu", fused=False)
        opt = make_optimizer(model, TrainConfig(optimizer="adamw", lr=0.01), only=dp.owned_ids())
        save_distributed_checkpoint(tmp / "ck", model, opt, None, dp, config={}, progress={"steps": 0},
                                    manifest_hash="0" * 64)
        dist.barrier()
        if rank == 0:
            f = tmp / "ck" / "rank-00001.pt"
            raw = bytearray(f.read_bytes())
            raw[len(raw) // 2] ^= 0xFF
            f.write_bytes(bytes(raw))
        dist.barrier()
        before = {k: v.clone() for k, v in model.state_dict().items()}
        with torch.no_grad():
            for p in model.parameters():
                p.add_(1.0)
        changed = {k: v.clone() for k, v in model.state_dict().items()}
        try:
            load_distributed_checkpoint(tmp / "ck", model, opt, None, dp)
        except ValueError as e:
            assert "checksum" in str(e), str(e)
            assert all(torch.equal(changed[k], v) for k, v in model.state_dict().items()), "state was installed"
            assert any(not torch.equal(before[k], v) for k, v in model.state_dict().items())
            print(f"SCENARIO_OK {scenario}", flush=True)
    elif scenario == "nonfinite":
        from tensor_train_ing_b200.config import Config
        from tensor_train_ing_b200.engine import TrainEngine
        torch.manual_seed(0)
        cfg = Config(model=ModelConfig(layers=1, d_model=16, heads=2, d_key=4, d_value=4, d_mlp=8, vocab_size=31,
                                       padded_vocab=32),
                     train=TrainConfig(optimizer="adamw", lr=0.01, grad_clip=1.0, compile=False, bf16_compute=False))
        eng = TrainEngine(cfg, device="cpu", micro_batch=2, model=TensorLM(cfg.model))
        g = torch.Generator().manual_seed(rank)
        idx = torch.randint(0, 31, (2, 8), generator=g)
        eng.begin_update()
        eng.forward_backward(idx, torch.zeros_like(idx), torch.roll(idx, -1, 1), torch.tensor(1.0 / 16))
        if rank == 1:
            with torch.no_grad():
                next(p for p in eng.model.parameters() if p.grad is not None).grad.view(-1)[0] = float("inf")
        before = {k: v.clone() for k, v in eng.model.state_dict().items()}
        try:
            eng.finish_update(error_if_nonfinite=True)
        except RuntimeError as e:
            assert "non-finite" in str(e), str(e)
            assert all(torch.equal(before[k], v) for k, v in eng.model.state_dict().items()), "weights changed"
            print(f"SCENARIO_OK {scenario}", flush=True)
    elif scenario == "disk_full":
        import shutil
        from collections import namedtuple
        torch.manual_seed(0)
        cfg = ModelConfig(layers=1, d_model=16, heads=2, d_key=4, d_value=4, d_mlp=8, vocab_size=31, padded_vocab=32)
        model = TensorLM(cfg)
        dp = ShardedDataParallel(model, "cpu", fused=False)
        opt = make_optimizer(model, TrainConfig(optimizer="adamw", lr=0.01), only=dp.owned_ids())
        if rank == 0:
            usage = namedtuple("usage", "total used free")
            shutil.disk_usage = lambda path: usage(10 ** 6, 10 ** 6 - 1024, 1024)
        try:
            save_distributed_checkpoint(tmp / "ck", model, opt, None, dp, config={}, progress={"steps": 0},
                                        manifest_hash="0" * 64)
        except ValueError as e:
            assert "bytes are free" in str(e), str(e)
            assert not (tmp / "ck").exists() and not any(tmp.glob(".ck.tmp-*"))
            print(f"SCENARIO_OK {scenario}", flush=True)
    elif scenario == "dead_rank":
        dist.barrier()
        if rank == 1:
            os._exit(0)  # leaves between steps, with no collective in flight
        try:
            t = torch.ones(4)
            dist.all_reduce(t)
        except Exception:  # noqa: BLE001 - gloo reports the lost peer or the timeout
            print(f"SCENARIO_OK {scenario}", flush=True)
            os._exit(0)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
