"""Worker (NCCL, one GPU per rank): the peer-memory reduce-scatter / all-gather of
ShardedDataParallel against NCCL's collectives on the same buffers, then a few training steps of
both paths.  Prints PEER_OK on rank 0."""
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


def batch(g, world, rank):
    idx = torch.randint(0, 1000, (4 * world, 256), generator=g)
    doc = torch.zeros_like(idx)
    doc[:, 100:] = 1
    tgt = torch.roll(idx, -1, 1)
    tgt[:, -1] = -100
    sl = slice(4 * rank, 4 * rank + 4)
    return idx[sl], doc[sl], tgt[sl]


def rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def main():
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    b = build(True)
    dp = b.dp
    g = torch.Generator().manual_seed(1)
    # ---- the collectives themselves against NCCL on the same data
    idx, doc, tgt = batch(g, world, rank)
    b.zero_grad()
    b.forward_backward(idx, doc, tgt, torch.ones((), device="cuda"))
    full = dp.grad_flat.clone()
    dist.all_reduce(full)  # the peer regions are packed (unequal): compare against an all-reduce
    expect = dp.region(full)
    dp.reduce_gradients()
    got = dp.region(dp.grad_flat)
    e_rs = rel(got, expect)
    e_sq = abs(float(dp._sq) - float(expect.double().square().sum())) / float(expect.double().square().sum())
    with torch.no_grad():
        dp.region(dp.param_flat).add_(0.25 * (rank + 1))
    pf = dp.param_flat.clone()
    want = pf.clone()
    for r in range(world):  # every rank region from its owner
        a, n = dp._rstart[r], dp._rlen[r]
        if n:
            dist.broadcast(want[a:a + n], src=r)
    for p in b.model.parameters():
        p.data.add_(0.0)  # bump versions like an optimizer step
    dp.gather_params()
    torch.cuda.synchronize()
    check_status()
    for kind, obj, params, off, n, owner in dp.units:  # alignment padding is not gathered
        assert torch.equal(dp.param_flat[off:off + n], want[off:off + n]), "peer all-gather differs from NCCL"
    assert e_rs < 1e-6 and e_sq < 1e-5, (e_rs, e_sq)
    for kind, obj, *_ in dp.units:
        if kind == "group":
            ref = torch.cat([p.detach().reshape(obj.rows[i], obj.d_in) for i, p in enumerate(obj.params)]).bfloat16()
            assert torch.equal(obj._cache, ref), "stale bf16 cache"
            assert obj._key == obj._version_key()
    # ---- training steps: peer path vs NCCL path
    del b
    a, b = build(False), build(True)
    for step in range(3):
        batch_ = batch(g, world, rank)
        la, _ = a.step(*batch_)
        lb, _ = b.step(*batch_)
        torch.cuda.synchronize()
        check_status()
        assert abs(float(la) - float(lb)) <= 1e-3 * abs(float(la)), (float(la), float(lb))
    for p in b.model.parameters():
        mine = p.detach().clone()
        dist.broadcast(p.detach(), src=0)
        assert torch.equal(mine, p.detach()), "peer all-gather left replicas different"
    if rank == 0:
        print(f"PEER_OK rs_rel={e_rs:.2e} sq_rel={e_sq:.2e}", flush=True)
    dist.barrier()
    del a, b
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
