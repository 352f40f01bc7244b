"""Worker: N-rank ShardedDataParallel TrainEngine steps == one process on the whole batch (fp64, gloo).

Run under torchrun; prints ``MAXERR <value>`` on rank 0."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig  # noqa: E402
from tensor_train_ing_b200.engine import TrainEngine  # noqa: E402
from tensor_train_ing_b200.models.model import TensorLM  # noqa: E402


def main():
    optimizer = sys.argv[1]
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.set_default_dtype(torch.float64)
    cfg = Config(model=ModelConfig(layers=2, d_model=16, heads=2, d_key=4, d_value=8, d_mlp=24, vocab_size=61,
                                   padded_vocab=64),
                 train=TrainConfig(optimizer=optimizer, lr=0.02, grad_clip=0.5))
    torch.manual_seed(0)
    ref_model = TensorLM(cfg.model)
    torch.manual_seed(0)
    model = TensorLM(cfg.model)
    ref = None
    if rank == 0:
        ref = TrainEngine(cfg, device="cpu", micro_batch=3, model=ref_model, group=dist.new_group([0]))
    else:
        dist.new_group([0])
    eng = TrainEngine(cfg, device="cpu", micro_batch=2, model=model)
    g = torch.Generator().manual_seed(1)
    rows, T = 4 * world, 12
    for step in range(3):
        idx = torch.randint(0, 61, (rows, T), generator=g)
        doc = torch.zeros(rows, T, dtype=torch.long)
        doc[:, 7:] = 1
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -100
        tgt[:, 6] = -100
        per = rows // world
        sl = slice(rank * per, (rank + 1) * per)
        loss, count = eng.step(idx[sl], doc[sl], tgt[sl])
        if rank == 0:
            rloss, rcount = ref.step(idx, doc, tgt)
            assert int(count) == int(rcount)
            # the engine accumulates the reported loss in fp32
            assert abs(float(loss) - float(rloss)) < 1e-6 * max(1.0, abs(float(rloss))), (float(loss), float(rloss))
    err = torch.zeros((), dtype=torch.float64)
    if rank == 0:
        for (n, a), (_, b) in zip(model.named_parameters(), ref_model.named_parameters()):
            err = torch.maximum(err, (a.detach() - b.detach()).abs().max())
    # every rank's replica must be identical to rank 0's
    for p in model.parameters():
        mine = p.detach().clone()
        dist.broadcast(p.detach(), src=0)
        assert torch.equal(mine, p.detach()), "replicas diverged"
    owned = len(eng.dp.owned_params())
    counts = [None] * world
    dist.all_gather_object(counts, owned)
    if rank == 0:
        assert sum(counts) == len([p for p in model.parameters() if p.requires_grad]), counts
        print(f"MAXERR {float(err):.3e}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
