"""Polynomial attention in chunked linear-state form (every kind, documents, padding, any chunk
size) against the dense oracle in fp64; the model's ``recurrent`` backend; and the context-parallel
split over gloo ranks."""
import os
import subprocess
import sys

import pytest
import torch

from tensor_train_ing_b200.config import ModelConfig
from tensor_train_ing_b200.models.attention import doc_positions, polynomial_attention, row_scale_mask, visible_mask
from tensor_train_ing_b200.models.long_context import chunked_polynomial_attention
from tensor_train_ing_b200.models.model import TensorLM

HERE = os.path.dirname(os.path.abspath(__file__))


def _docs(B=2, T=70):
    docs = torch.zeros(B, T, dtype=torch.long)
    docs[0, 20:] = 1
    docs[0, 45:] = 2
    docs[1, :] = 5
    docs[1, T - 10:] = -torch.arange(1, 11)
    return docs


@pytest.mark.parametrize("kind", ["signed_product", "offset_square", "lower_degree_mix"])
@pytest.mark.parametrize("chunk", [1, 7, 64, 256])
def test_chunked_form_equals_dense_attention(kind, chunk):
    torch.manual_seed(0)
    docs = _docs()
    B, T = docs.shape
    q1, k1, q2, k2, v = (torch.randn(B, 3, T, 4, dtype=torch.float64, requires_grad=True) for _ in range(5))
    coef, b = torch.randn(3, 4, dtype=torch.float64), torch.randn(3, dtype=torch.float64)
    two = kind != "offset_square"
    want = polynomial_attention(kind, q1, k1, q2 if two else None, k2 if two else None, v,
                                row_scale_mask(visible_mask(docs), 0.5, dtype=torch.float64), coef=coef, b=b)
    scale = torch.where(docs >= 0, (doc_positions(docs) + 1).double().pow(-0.5), 0.0)
    got, _, _ = chunked_polynomial_attention(kind, q1, k1, q2, k2, v, docs, scale, chunk=chunk, coef=coef, b=b)
    torch.testing.assert_close(got, want, rtol=1e-10, atol=1e-12)
    gy = torch.randn_like(want)
    g1 = torch.autograd.grad(want, [q1, k1, v], gy)
    g2 = torch.autograd.grad(got, [q1, k1, v], gy)
    for a, c in zip(g1, g2):
        torch.testing.assert_close(c, a, rtol=1e-9, atol=1e-11)


def test_recurrent_backend_matches_the_dense_module_path():
    kw = dict(layers=2, d_model=32, heads=2, d_key=8, d_value=16, d_mlp=48, vocab_size=97, padded_vocab=128)
    torch.manual_seed(0)
    dense = TensorLM(ModelConfig(**kw, attention_backend="reference")).double().eval()
    recurrent = TensorLM(ModelConfig(**kw, attention_backend="recurrent")).double().eval()
    recurrent.load_state_dict(dense.state_dict())
    idx = torch.randint(0, 97, (2, 70))
    docs = _docs()
    # the dense path builds its row-scale mask in fp32, the recurrent one its scales in fp64
    torch.testing.assert_close(recurrent(idx, doc_ids=docs), dense(idx, doc_ids=docs), rtol=1e-5, atol=1e-7)
    with pytest.raises(AssertionError):  # config validation fails the way the schema's other rules do
        ModelConfig(**kw, attention="softmax", attention_backend="recurrent")


@pytest.mark.slow
@pytest.mark.parametrize("kind", ["signed_product", "offset_square"])
def test_context_parallel_attention_equals_whole_row_attention(kind):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
           "--nproc-per-node", "3", os.path.join(HERE, "dist_workers", "context_parallel.py"), kind]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-4000:]
    assert "CP_OK" in out.stdout
