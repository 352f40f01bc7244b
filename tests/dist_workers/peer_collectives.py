"""Worker (NCCL, one GPU per rank): the peer-memory reduce-scatter / all-gather path of
ShardedDataParallel against the NCCL path on identical training steps.  Prints PEER_OK on rank 0."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig  # noqa: E402
from tensor_train_ing_b200.engine import TrainEngine  # noqa: E402
from tensor_train_ing_b200.ops._ext import check_status  # noqa: E402


def build(peer: bool):
    os.environ["TTB_PEER_COLLECTIVES"] = "1" if peer else "0"
    cfg = Config(model=ModelConfig(layers=2, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                                   padded_vocab=1024, loss_chunk_tokens=512),
                 train=TrainConfig(optimizer="muon", lr=0.01, aux_adamw_lr=0.003, grad_clip=0.5))
    torch.manual_seed(0)
    eng = TrainEngine(cfg, device="cuda", micro_batch=2)
    assert eng.dp.peer == peer
    return eng


def main():
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    a, b = build(False), build(True)
    g = torch.Generator().manual_seed(1)
    for step in range(3):
        idx = torch.randint(0, 1000, (4 * world, 256), generator=g)
        doc = torch.zeros_like(idx)
        doc[:, 100:] = 1
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -100
        sl = slice(4 * rank, 4 * rank + 4)
        la, _ = a.step(idx[sl], doc[sl], tgt[sl])
        lb, _ = b.step(idx[sl], doc[sl], tgt[sl])
        torch.cuda.synchronize()
        check_status()
        assert abs(float(la) - float(lb)) <= 1e-3 * abs(float(la)), (float(la), float(lb))
    worst = 0.0
    for (n, pa), (_, pb) in zip(a.model.named_parameters(), b.model.named_parameters()):
        worst = max(worst, float((pa.detach() - pb.detach()).abs().max() / pa.detach().abs().max().clamp_min(1e-12)))
    assert worst < 2e-2, worst  # reduction order differs (NCCL ring vs rank order); Muon amplifies little
    # replicas of the peer path are bitwise identical across ranks
    for p in b.model.parameters():
        mine = p.detach().clone()
        dist.broadcast(p.detach(), src=0)
        assert torch.equal(mine, p.detach()), "peer all-gather left replicas different"
    # the fused all-gather wrote the bf16 operand caches from the gathered fp32 values
    for kind, obj, *_ in b.dp.units:
        if kind == "group":
            ref = torch.cat([p.detach().reshape(obj.rows[i], obj.d_in) for i, p in enumerate(obj.params)]).bfloat16()
            assert torch.equal(obj._cache, ref), "stale bf16 cache"
            assert obj._key == obj._version_key()
    if rank == 0:
        print(f"PEER_OK worst_rel={worst:.3e}", flush=True)
    dist.barrier()
    del a, b
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
