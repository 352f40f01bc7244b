"""Worker (NCCL, one GPU per rank): parameter-sharded training on the fused path (fp32 masters only
on owners, bf16 caches gathered from them, per-block gradient reduction through peer memory or
NCCL) against the replicated layout.  Prints SHARD_OK on rank 0."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig  # noqa: E402
from tensor_train_ing_b200.engine import TrainEngine  # noqa: E402
from tensor_train_ing_b200.ops._ext import check_status  # noqa: E402

CFG = Config(model=ModelConfig(layers=3, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                               padded_vocab=1024, loss_chunk_tokens=512),
             train=TrainConfig(optimizer="muon", lr=0.01, aux_adamw_lr=0.003, grad_clip=0.5))


def build(shard: bool, peer: bool, gather: bool = True):
    os.environ["TTB_PEER_COLLECTIVES"] = "1" if peer else "0"
    os.environ["TTB_FUSED_GATHER"] = "1" if gather else "0"
    torch.manual_seed(0)
    eng = TrainEngine(CFG, device="cuda", micro_batch=2, shard_params=shard)
    assert eng.dp.peer == peer and eng.dp.shard_params == shard
    assert eng.dp.fused_gather == (shard and peer and gather)
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
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def main():
    dist.init_process_group("nccl")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    engines = {"replicated": build(False, True), "sharded_gather": build(True, True),
               "sharded_peer": build(True, True, gather=False), "sharded_nccl": build(True, False)}
    sharded = ("sharded_gather", "sharded_peer", "sharded_nccl")
    ref = engines["replicated"]
    ref_state = {k: v.detach().cpu() for k, v in ref.model.state_dict().items()}
    for name in sharded:
        eng = engines[name]
        dp = eng.dp
        assert dp.model._ttb_weights_remote
        owned = sum(su.n for su in dp.sunits if su.owner == rank)
        total = sum(su.n for su in dp.sunits)
        assert owned < total, "a rank holds every sharded master"
        full = dp.full_state_dict(dst=None)
        for k, v in ref_state.items():  # the streamed initialisation is the serial one, bit for bit
            assert torch.equal(full[k], v), f"{name}: initial {k} differs"
        for su in dp.sunits:  # every rank's bf16 operands come from the owners' masters
            want = torch.cat([ref_state[n].reshape(-1) for n in su.names]).to("cuda").bfloat16()
            if dp.fused_gather:
                # no full copy on any rank: this rank's row shard, and the rows gathered from both ranks
                assert su.group._cache is None, f"{name}: a full bf16 copy of {su.names[0]}"
                lo, hi = su.cuts[rank], su.cuts[rank + 1]
                mine = dp.wshard[su.woff:su.woff + (hi - lo) * su.cols]
                assert torch.equal(mine, want[lo * su.cols:hi * su.cols]), f"{name}: row shard of {su.names[0]}"
                assert torch.equal(su.group.bf16().reshape(-1), want), f"{name}: gathered {su.names[0]}"
            else:
                assert torch.equal(su.group._cache.reshape(-1), want), f"{name}: cache of {su.names[0]}"
    g = torch.Generator().manual_seed(1)
    losses = {k: [] for k in engines}
    for step in range(3):
        idx, doc, tgt = batch(g, world, rank)
        for name, eng in engines.items():
            loss, count = eng.step(idx, doc, tgt)
            losses[name].append(float(loss) / float(count))
    torch.cuda.synchronize()
    check_status()
    final = {k: v.detach().cpu() for k, v in ref.model.state_dict().items()}
    window = engines["sharded_gather"].dp.window
    assert window.gathers > 0
    if rank == 0:
        print(f"sharded_gather: {window.gathers} gathers, window {window.nbytes / 2**20:.1f} MiB, "
              f"row shards {engines['sharded_gather'].dp.wshard.numel() * 2 / 2**20:.1f} MiB", flush=True)
    for name in sharded:
        for a, b in zip(losses[name], losses["replicated"]):
            assert abs(a - b) < 1e-3 * abs(b), (name, losses[name], losses["replicated"])
        full = engines[name].dp.full_state_dict(dst=None)
        worst = max(rel(full[k], final[k]) for k in final if final[k].is_floating_point())
        assert worst < 2e-2, (name, worst)
        if rank == 0:
            print(f"{name}: losses {losses[name]} max param rel diff {worst:.2e}", flush=True)
    if rank == 0:
        print("SHARD_OK", flush=True)
    del engines
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
