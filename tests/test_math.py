"""CPU fp64 oracle tests of the model math (reference tests/test_math.py covers the same facts)."""
import math

import pytest
import torch
import torch.nn.functional as F

from helpers import TINY_MODEL
from tensor_train_ing_b200.config import ModelConfig
from tensor_train_ing_b200.models.attention import (doc_positions, polynomial_attention,
                                                    polynomial_attention_recurrent, row_scale_mask,
                                                    row_scale_vector, visible_mask)
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.models.normalization import (GroupRMSNorm, LaggedRMS, RMSNorm, SpectralLinear,
                                                        freeze_spectral, rms_jacobian)
from tensor_train_ing_b200.ops.linear_ce import chunked_linear_cross_entropy_reference


@pytest.fixture(autouse=True)
def _fp64():
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    torch.manual_seed(0)
    yield
    torch.set_default_dtype(prev)


def _model(**kw):
    cfg = ModelConfig(**{**TINY_MODEL, **kw})
    return TensorLM(cfg).double().eval()


def test_rms_jacobian_matches_autograd():
    x, g = torch.randn(12), torch.rand(12) + .5
    norm = RMSNorm(12, 1e-6).double()
    with torch.no_grad():
        norm.weight.copy_(g)
    J = torch.autograd.functional.jacobian(norm, x)
    torch.testing.assert_close(J, rms_jacobian(x, g, 1e-6), rtol=1e-10, atol=1e-12)


def test_group_rms_is_block_diagonal_dependency():
    norm = GroupRMSNorm(16, groups=4).double()
    J = torch.autograd.functional.jacobian(norm, torch.randn(16))
    for i in range(4):
        for j in range(4):
            block = J[4 * i:4 * i + 4, 4 * j:4 * j + 4]
            assert (block.abs().max() > 0) == (i == j)


@pytest.mark.parametrize("kind", ["signed_product", "offset_square", "lower_degree_mix"])
def test_attention_gradcheck(kind):
    B, H, T, dk, dv = 1, 2, 5, 3, 2
    doc = torch.tensor([[0, 0, 1, 1, 1]])
    C = row_scale_mask(visible_mask(doc), 1.0, torch.float64)
    q1, k1, q2, k2 = (torch.randn(B, H, T, dk, requires_grad=True) for _ in range(4))
    v = torch.randn(B, H, T, dv, requires_grad=True)
    coef = torch.randn(H, 4, requires_grad=True)
    b = torch.randn(H, requires_grad=True)
    fn = lambda *a: polynomial_attention(kind, *a[:5], C, coef=a[5], b=a[6])  # noqa: E731
    assert torch.autograd.gradcheck(fn, (q1, k1, q2, k2, v, coef, b))


def test_recurrent_equals_direct():
    H, T, dk, dv = 2, 7, 4, 3
    q1, k1, q2, k2 = (torch.randn(H, T, dk) for _ in range(4))
    v = torch.randn(H, T, dv)
    doc = torch.zeros(1, T, dtype=torch.long)
    scale = row_scale_vector(doc, 1.0)[0]
    C = row_scale_mask(visible_mask(doc), 1.0, torch.float64)
    direct = polynomial_attention("signed_product", q1[None], k1[None], q2[None], k2[None], v[None], C)[0]
    torch.testing.assert_close(polynomial_attention_recurrent(q1, k1, q2, k2, v, scale), direct)


def test_masked_entries_zero_after_polynomial():
    # (S + b)^2 is positive everywhere; masking before the polynomial would leak b^2 into hidden keys
    B, H, T, d = 1, 1, 4, 2
    q, k, v = torch.randn(B, H, T, d), torch.randn(B, H, T, d), torch.randn(B, H, T, d)
    doc = torch.zeros(1, T, dtype=torch.long)
    C = visible_mask(doc).double()
    b = torch.tensor([3.0])
    y = polynomial_attention("offset_square", q, k, None, None, v, C, b=b)
    S = q @ k.transpose(-1, -2) / math.sqrt(d)
    expected = (torch.tril(torch.ones(T, T)) * (S + 3.0) ** 2) @ v
    torch.testing.assert_close(y, expected)


def test_row_scale_vector_matches_mask():
    doc = torch.tensor([[0, 0, 0, 1, 1, -1, -2]])
    vis = visible_mask(doc)
    for p in (0.5, 1.0, 2.0):
        dense = row_scale_mask(vis, p, torch.float64)
        vec = row_scale_vector(doc, p)
        torch.testing.assert_close(dense.amax(-1)[0, 0], vec[0].double())
    assert doc_positions(doc).tolist() == [[0, 1, 2, 0, 1, 0, 0]]


@pytest.mark.parametrize("attention", ["signed_product", "offset_square", "lower_degree_mix", "softmax"])
def test_causal_prefix_invariance(attention):
    m = _model(attention=attention)
    idx = torch.randint(0, 97, (1, 9))
    full = m(idx)
    prefix = m(idx[:, :5])
    torch.testing.assert_close(full[:, :5], prefix, rtol=1e-9, atol=1e-10)


def test_document_isolation_and_position_reset():
    m = _model()
    a, b = torch.randint(0, 97, (1, 4)), torch.randint(0, 97, (1, 5))
    packed = m(torch.cat([a, b], 1), doc_ids=torch.tensor([[0] * 4 + [1] * 5]))
    alone = m(b, doc_ids=torch.zeros(1, 5, dtype=torch.long))
    torch.testing.assert_close(packed[:, 4:], alone, rtol=1e-9, atol=1e-10)


def test_padding_values_do_not_affect_real_tokens():
    m = _model()
    idx = torch.randint(0, 97, (1, 8))
    doc = torch.tensor([[0, 0, 0, 0, 0, -1, -2, -3]])
    y1 = m(idx, doc_ids=doc)
    idx2 = idx.clone()
    idx2[:, 5:] = torch.randint(0, 97, (1, 3))
    y2 = m(idx2, doc_ids=doc)
    torch.testing.assert_close(y1[:, :5], y2[:, :5], rtol=1e-12, atol=1e-12)


def test_padding_is_not_a_shared_document():
    # two padding tokens with distinct negative ids never see each other
    vis = visible_mask(torch.tensor([[0, -1, -2]]))
    assert not vis[0, 0, 1:].any() and not vis[0, 0, :, 1:].any()


def test_lagged_uses_previous_statistic_and_commits_once():
    n = LaggedRMS(4, eps=0.0, half_life_tokens=4.0).double()
    x = torch.full((2, 4), 2.0)
    n.collecting = True
    y = n(x)
    torch.testing.assert_close(y, x)  # initial mean_sq = 1: output is x, not x / 2
    assert float(n.commit(distributed=False)) == pytest.approx(4.0)  # first commit copies
    n.collecting = True
    n(torch.full((2, 4), 4.0))  # mean square 16, 2 tokens
    keep = 0.5 ** (2 / 4.0)
    assert float(n.commit(distributed=False)) == pytest.approx(keep * 4 + (1 - keep) * 16)
    assert float(n.commit(distributed=False)) == pytest.approx(keep * 4 + (1 - keep) * 16)  # nothing new


def test_lagged_excludes_padding():
    n = LaggedRMS(2, eps=0.0).double()
    n.collecting = True
    n.set_valid_mask(torch.tensor([True, False]))
    n(torch.tensor([[1.0, 1.0], [100.0, 100.0]]))
    assert float(n.commit(distributed=False)) == pytest.approx(1.0)


def test_spectral_effective_weight_reproduces_logits():
    m = _model(normalization="spectral_rms")
    idx = torch.randint(0, 97, (2, 6))
    before = m(idx)
    assert freeze_spectral(m) > 0
    torch.testing.assert_close(m(idx), before, rtol=1e-10, atol=1e-10)


def test_spectral_zero_weight_is_finite_and_zero():
    s = SpectralLinear(4, 3).double()
    with torch.no_grad():
        s.weight.zero_()
    s._power_step()
    y = s(torch.randn(5, 4))
    assert torch.isfinite(y).all() and (y == 0).all()


def test_chunked_ce_matches_full_cross_entropy_and_grads():
    x = torch.randn(13, 8, requires_grad=True)
    w = torch.randn(11, 8, requires_grad=True)
    t = torch.randint(0, 11, (13,))
    t[3] = -100
    loss = chunked_linear_cross_entropy_reference(x, w, t, chunk=4)
    ref = F.cross_entropy(x @ w.t(), t, reduction="sum", ignore_index=-100)
    torch.testing.assert_close(loss, ref)
    gx, gw = torch.autograd.grad(loss, (x, w))
    rx, rw = torch.autograd.grad(ref, (x, w))
    torch.testing.assert_close(gx, rx)
    torch.testing.assert_close(gw, rw)


def test_model_loss_chunking_matches_unchunked():
    m = _model()
    m2 = _model(loss_chunk_tokens=5)
    m2.load_state_dict(m.state_dict())
    idx = torch.randint(0, 97, (2, 6))
    t = torch.roll(idx, -1, 1)
    _, l1, _ = m(idx, targets=t, reduction="sum")
    _, l2, _ = m2(idx, targets=t, reduction="sum")
    torch.testing.assert_close(l1, l2)
    g1 = torch.autograd.grad(l1, list(m.parameters()), allow_unused=True)
    g2 = torch.autograd.grad(l2, list(m2.parameters()), allow_unused=True)
    for a, b in zip(g1, g2):
        if a is not None:
            torch.testing.assert_close(a, b)


def test_operator_audit_and_param_counts():
    m = _model()
    audit = m.operator_audit()
    assert audit["class"] in ("P", "N", "G")
    counts = m.param_counts()
    assert counts["total"] == sum(p.numel() for p in m.parameters())
    assert counts["matrices"] + counts["small"] == counts["total"]


def test_analysis_modes_cannot_leak_into_training():
    norm = RMSNorm(4, 1e-6).double()
    norm.denom_mode = "record"
    with pytest.raises(RuntimeError):
        norm(torch.randn(2, 4))
    norm.eval()
    norm(torch.randn(2, 4))
    assert norm.denom_saved is not None


def test_weight_cache_follows_fused_optimizer_steps():
    """torch's fused AdamW updates parameters without bumping their version counters; the bf16
    operand cache of a weight group must still be rebuilt after the step."""
    import torch
    from tensor_train_ing_b200.ops.weights import WeightGroup
    w = torch.nn.Parameter(torch.randn(16, 8))
    grp = WeightGroup([w])
    before = grp.bf16().clone()
    assert torch.equal(before, w.detach().bfloat16())
    w.grad = torch.randn(16, 8)
    opt = torch.optim.AdamW([w], lr=0.1, fused=True)
    v = w._version
    opt.step()
    assert w._version == v  # the case this guards against
    assert torch.equal(grp.bf16(), w.detach().bfloat16())
    assert not torch.equal(grp.bf16(), before)
