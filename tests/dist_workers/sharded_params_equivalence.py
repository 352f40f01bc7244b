"""Worker: parameter-sharded TrainEngine (fp32 masters only on owners, model built from the streamed
serial initialisation) == one process on the whole batch (fp64, gloo); then a sharded checkpoint
round trip continues identically.

Run under torchrun; prints ``MAXERR <value>`` and ``RESUMEERR <value>`` on rank 0."""
import os
import sys
import tempfile

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig  # noqa: E402
from tensor_train_ing_b200.distributed_checkpoint import (load_distributed_checkpoint,  # noqa: E402
                                                          save_distributed_checkpoint)
from tensor_train_ing_b200.engine import TrainEngine  # noqa: E402
from tensor_train_ing_b200.models.model import TensorLM  # noqa: E402


def batch(g, rows, T):
    idx = torch.randint(0, 61, (rows, T), generator=g)
    doc = torch.zeros(rows, T, dtype=torch.long)
    doc[:, 7:] = 1
    tgt = torch.roll(idx, -1, 1)
    tgt[:, -1] = -100
    tgt[:, 6] = -100
    return idx, doc, tgt


def main():
    optimizer, ckpt_root = sys.argv[1], sys.argv[2]
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.set_default_dtype(torch.float64)
    cfg = Config(model=ModelConfig(layers=3, d_model=16, heads=2, d_key=4, d_value=8, d_mlp=24, vocab_size=61,
                                   padded_vocab=64),
                 train=TrainConfig(optimizer=optimizer, lr=0.02, grad_clip=0.5))
    torch.manual_seed(0)
    ref_model = TensorLM(cfg.model)
    ref = None
    if rank == 0:
        ref = TrainEngine(cfg, device="cpu", micro_batch=3, model=ref_model, group=dist.new_group([0]),
                          shard_params=False)
    else:
        dist.new_group([0])
    torch.manual_seed(0)
    eng = TrainEngine(cfg, device="cpu", micro_batch=2, shard_params=True)  # meta model, streamed init
    assert eng.dp.shard_params and eng.dp.sunits
    owned = [su for su in eng.dp.sunits if su.owner == rank]
    assert len(eng.dp.sp_param) >= sum(su.n for su in owned)
    g = torch.Generator().manual_seed(1)
    rows, T = 4 * world, 12
    per = rows // world
    sl = slice(rank * per, (rank + 1) * per)
    for step in range(3):
        idx, doc, tgt = batch(g, rows, T)
        loss, count = eng.step(idx[sl], doc[sl], tgt[sl])
        if rank == 0:
            rloss, rcount = ref.step(idx, doc, tgt)
            assert int(count) == int(rcount)
            assert abs(float(loss) - float(rloss)) < 1e-6 * max(1.0, abs(float(rloss))), (float(loss), float(rloss))
    full = eng.dp.full_state_dict(dst=0)
    err = torch.zeros((), dtype=torch.float64)
    if rank == 0:
        ref_state = ref_model.state_dict()
        assert set(full) == set(ref_state), set(full) ^ set(ref_state)
        for k, v in ref_state.items():
            err = torch.maximum(err, (full[k] - v).abs().max())
        print(f"MAXERR {float(err):.3e}", flush=True)

    # sharded checkpoint round trip: a fresh sharded engine resumes and continues identically
    box = [tempfile.mkdtemp(dir=ckpt_root) if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    path = os.path.join(box[0], "ckpt")
    save_distributed_checkpoint(path, eng.model, eng.optimizer, None, eng.dp, config={"t": 1}, progress={"s": 3},
                                manifest_hash="h")
    torch.manual_seed(123)  # a different init: everything must come from the checkpoint
    eng2 = TrainEngine(cfg, device="cpu", micro_batch=2, shard_params=True)
    load_distributed_checkpoint(path, eng2.model, eng2.optimizer, None, eng2.dp, restore_rng=False)
    eng2.dp.gather_params()
    idx, doc, tgt = batch(g, rows, T)
    l1, _ = eng.step(idx[sl], doc[sl], tgt[sl])
    l2, _ = eng2.step(idx[sl], doc[sl], tgt[sl])
    a, b = eng.dp.full_state_dict(dst=0), eng2.dp.full_state_dict(dst=0)
    if rank == 0:
        rerr = max(float((a[k] - b[k]).abs().max()) for k in a)
        rerr = max(rerr, abs(float(l1) - float(l2)))
        print(f"RESUMEERR {rerr:.3e}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
