"""Peer-memory collectives on 2 GPUs against NCCL (skipped with fewer than two GPUs)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_reduce_scatter_and_all_gather_match_nccl():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--standalone",
           "--local-addr", "127.0.0.1", "--nproc-per-node", "2", os.path.join(HERE, "dist_workers", "peer_collectives.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=660, env=env)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-4000:]
    assert "PEER_OK" in out.stdout


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_parameter_sharded_training_matches_replicated():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--standalone",
           "--local-addr", "127.0.0.1", "--nproc-per-node", "2",
           os.path.join(HERE, "dist_workers", "sharded_params_gpu.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=660, env=env)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-4000:]
    assert "SHARD_OK" in out.stdout


def test_parameter_sharded_single_gpu_matches_replicated():
    """One rank owns every unit: the staging / accumulation / cache-gather path against the
    replicated engine.  Same kernels and the same summation order per micro-batch, and no clipping
    (whose norm is summed over differently split buffers), so training is bitwise identical."""
    from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
    from tensor_train_ing_b200.engine import TrainEngine
    from tensor_train_ing_b200.ops._ext import check_status
    cfg = Config(model=ModelConfig(layers=2, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                                   padded_vocab=1024, loss_chunk_tokens=512),
                 train=TrainConfig(optimizer="muon", lr=0.01, aux_adamw_lr=0.003, grad_clip=1e9))
    torch.manual_seed(0)
    ref = TrainEngine(cfg, device="cuda", micro_batch=2, shard_params=False)
    torch.manual_seed(0)
    eng = TrainEngine(cfg, device="cuda", micro_batch=2, shard_params=True)
    assert eng.dp.shard_params and len(eng.dp.buckets) == cfg.model.layers + 1
    g = torch.Generator().manual_seed(1)

    def batch():
        idx = torch.randint(0, 1000, (4, 256), generator=g)
        doc = torch.zeros_like(idx)
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -100
        return idx, doc, tgt

    # gradients of two micro-batches: staged, reduced and accumulated == accumulated in the GEMMs
    inv = torch.ones((), device="cuda")
    idx, doc, tgt = batch()
    for e in (ref, eng):
        e.zero_grad()
        e.forward_backward(idx, doc, tgt, inv)
        e.dp.reduce_gradients()
    mine = dict(eng.model.named_parameters())
    for name, p in ref.model.named_parameters():
        assert torch.equal(p.grad, mine[name].grad), name
    for _ in range(3):
        idx, doc, tgt = batch()
        l1, c1 = ref.step(idx, doc, tgt)
        l2, c2 = eng.step(idx, doc, tgt)
        assert float(l1) == float(l2)
    torch.cuda.synchronize()
    check_status()
    a = ref.model.state_dict()
    b = eng.dp.full_state_dict(dst=None)
    for k, v in a.items():
        assert torch.equal(b[k], v.cpu()), k


def test_parameter_sharded_single_gpu_with_fused_gather_matches_replicated(monkeypatch):
    """The fused all-gather path on one rank: the sharded groups' bf16 rows live only in the row-shard
    buffer (no full cache), every forward GEMM gathers its weight into a window slot itself and the
    other consumers find it resident or gather it alone.  The staged values equal the caches' values
    and the kernels' arithmetic is unchanged, so training is bitwise identical to the replicated
    engine."""
    from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
    from tensor_train_ing_b200.engine import TrainEngine
    from tensor_train_ing_b200.ops._ext import check_status
    cfg = Config(model=ModelConfig(layers=2, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                                   padded_vocab=1024, loss_chunk_tokens=512),
                 train=TrainConfig(optimizer="muon", lr=0.01, aux_adamw_lr=0.003, grad_clip=1e9))
    torch.manual_seed(0)
    ref = TrainEngine(cfg, device="cuda", micro_batch=2, shard_params=False)
    monkeypatch.setenv("TTB_FUSED_GATHER", "1")
    monkeypatch.setenv("TTB_GATHER_SLOTS", "3")  # fewer slots than a block's groups: evictions and re-gathers
    torch.manual_seed(0)
    eng = TrainEngine(cfg, device="cuda", micro_batch=2, shard_params=True)
    assert eng.dp.fused_gather and all(su.group._cache is None for su in eng.dp.sunits)
    g = torch.Generator().manual_seed(1)
    for _ in range(3):
        idx = torch.randint(0, 1000, (4, 256), generator=g)
        doc = torch.zeros_like(idx)
        doc[:, 130:] = 1
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -100
        l1, _ = ref.step(idx, doc, tgt)
        l2, _ = eng.step(idx, doc, tgt)
        assert float(l1) == float(l2)
    torch.cuda.synchronize()
    check_status()
    assert eng.dp.window.gathers > 3 * 2 * cfg.model.layers
    assert all(su.group._cache is None for su in eng.dp.sunits)
    a = ref.model.state_dict()
    b = eng.dp.full_state_dict(dst=None)
    for k, v in a.items():
        assert torch.equal(b[k], v.cpu()), k
