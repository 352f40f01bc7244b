"""Rows without a scored target are dropped from a micro-batch before the forward pass
(tensor_train_ing_b200/train.py `_trim_unscored_rows`; reference tnlm/train.py row trimming).  Rows
are independent sequences, so the summed loss, the scored-token count and every parameter gradient
must be the same with and without them (CPU)."""
import copy

import pytest
import torch

from tensor_train_ing_b200.config import ModelConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.train import _trim_unscored_rows


def _batch():
    g = torch.Generator().manual_seed(4)
    idx = torch.randint(0, 40, (5, 6), generator=g)
    docs = torch.tensor([[0, 0, 0, 1, 1, 1],
                         [0, 0, 0, 0, 0, 0],         # no scored target: dropped
                         [0, 0, 1, 1, 1, -1],        # trailing padding
                         [-1, -2, -3, -4, -5, -6],   # all padding: dropped
                         [0, 0, 0, 0, 0, 0]])
    targets = torch.randint(0, 40, (5, 6), generator=g)
    targets[docs < 0] = -100
    targets[1] = -100
    targets[0, 2] = -100  # a document's last token predicts nothing
    targets[4, :3] = -100
    return idx, docs, targets


@pytest.mark.parametrize("normalization", ["pre_rms", "group_rms", "spectral_rms"])
@pytest.mark.parametrize("attention", ["signed_product", "softmax"])
@pytest.mark.parametrize("chunk", [0, 3])
def test_trimmed_batch_gives_the_same_loss_and_gradients(normalization, attention, chunk):
    torch.manual_seed(0)
    cfg = ModelConfig(layers=2, d_model=16, heads=2, d_key=8, d_value=8, d_mlp=24, vocab_size=40, padded_vocab=64,
                      attention=attention, normalization=normalization, loss_chunk_tokens=chunk)
    full_model = TensorLM(cfg)
    trim_model = copy.deepcopy(full_model)
    idx, docs, targets = _batch()
    t_idx, t_docs, t_targets = _trim_unscored_rows(idx, docs, targets, enabled=True)
    assert t_idx.shape[0] == 3 and torch.equal(t_targets, targets[[0, 2, 4]])
    results = []
    for model, batch in ((full_model, (idx, docs, targets)), (trim_model, (t_idx, t_docs, t_targets))):
        model.train()
        _, loss, n = model(batch[0], batch[1], batch[2], reduction="sum")
        loss.backward()
        results.append((loss.detach(), int(n), {k: p.grad.clone() for k, p in model.named_parameters()
                                                if p.grad is not None}))
    (lf, nf, gf), (lt, nt, gt) = results
    assert nf == nt == int((targets != -100).sum())
    torch.testing.assert_close(lt, lf, rtol=1e-5, atol=1e-6)
    assert gf.keys() == gt.keys() and len(gf) == sum(1 for _ in full_model.parameters())
    for k in gf:
        torch.testing.assert_close(gt[k], gf[k], rtol=1e-4, atol=1e-6, msg=k)


def test_row_buckets_keep_a_few_sizes_by_retaining_unscored_rows_in_order():
    idx = torch.arange(8 * 3).view(8, 3)
    docs = torch.zeros(8, 3, dtype=torch.long)
    targets = torch.full((8, 3), -100)
    for r in (1, 4, 6):
        targets[r, 0] = 5
    # three scored rows of eight: the bucket sizes are 1, 2, 4, 8, so one unscored row (the first) stays
    i, _, t = _trim_unscored_rows(idx, docs, targets, enabled=True, bucket_rows=True)
    assert i[:, 0].tolist() == [0, 3, 12, 18] and int((t != -100).sum()) == 3
    i, _, _ = _trim_unscored_rows(idx, docs, targets, enabled=True)
    assert i[:, 0].tolist() == [3, 12, 18]
    targets[[0, 2, 3]] = 5  # six scored rows: the bucket is the whole batch
    i, _, _ = _trim_unscored_rows(idx, docs, targets, enabled=True, bucket_rows=True)
    assert i.shape[0] == 8
    none = torch.full((8, 3), -100)
    assert _trim_unscored_rows(idx, docs, none, enabled=True, bucket_rows=True)[0].shape[0] == 0
    assert _trim_unscored_rows(idx, docs, none, enabled=False)[0].shape[0] == 8
