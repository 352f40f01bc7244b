"""sm_100a kernels vs plain PyTorch fp32/fp64 references of the same op (tolerances fixed up
front, as in the reference's kernel acceptance tests: bf16 relative error < 3e-2)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from tensor_train_ing_b200.models.attention import (apply_rope, polynomial_attention, rope_tables, row_scale_mask,
                                                    row_scale_vector, visible_mask, doc_positions)
from tensor_train_ing_b200.ops import fused
from tensor_train_ing_b200.ops._ext import lib


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def make_docs(B, T, seed=0, pad=True):
    g = torch.Generator().manual_seed(seed)
    docs = torch.empty(B, T, dtype=torch.long)
    for b in range(B):
        t, d = 0, 0
        while t < T:
            n = int(torch.randint(5, max(6, T // 2), (1,), generator=g))
            docs[b, t:t + n] = d
            t += n
            d += 1
        if pad and b == B - 1:
            docs[b, T - 7:] = -torch.arange(1, 8)  # unique negative ids = padding
    return docs


def dense_attention(kind, qkv, cols, B, T, H, dk, dv, docs, power, kpar):
    def head(c, d):
        return qkv[:, c:c + H * d].double().view(B, T, H, d).transpose(1, 2)
    q1, k1 = head(cols[0], dk), head(cols[1], dk)
    q2, k2 = (head(cols[2], dk), head(cols[3], dk)) if kind != "offset_square" else (None, None)
    v = head(cols[4], dv)
    C = row_scale_mask(visible_mask(docs), power, dtype=torch.float64)
    coef = kpar.double() if kind == "lower_degree_mix" else None
    b = kpar.double() if kind == "offset_square" else None
    y = polynomial_attention(kind, q1, k1, q2, k2, v, C, coef=coef, b=b)
    return y.transpose(1, 2).reshape(B * T, H * dv)


@pytest.mark.parametrize("kind", ["signed_product", "offset_square", "lower_degree_mix"])
@pytest.mark.parametrize("dk", [64, 128])
@pytest.mark.parametrize("B,T", [(2, 200), (1, 77), (1, 384)])
def test_poly_attention_fwd_bwd(kind, dk, B, T):
    check_poly_attention(kind, dk, B, T, H=2)


@pytest.mark.parametrize("kind", ["signed_product", "offset_square", "lower_degree_mix"])
@pytest.mark.parametrize("limit", [1, 3])
def test_poly_attention_persistent_ctas_work_through_many_tiles(kind, limit):
    """The persistent kernels with 1 or 3 CTAs: each CTA takes tiles of different lengths (causal,
    document starts) one after another through the same rings and accumulators."""
    lib().attn_grid_limit(limit)
    try:
        check_poly_attention(kind, 128, 2, 520, H=3)
    finally:
        lib().attn_grid_limit(0)


def test_poly_attention_more_tiles_than_sms():
    check_poly_attention("signed_product", 128, 3, 1100, H=6)  # 3 * 6 * 9 = 162 query tiles


def check_poly_attention(kind, dk, B, T, H):
    torch.manual_seed(0)
    dv = dk
    dev = "cuda"
    nqk = 4 if kind != "offset_square" else 2
    cols = [0, H * dk, 2 * H * dk, 3 * H * dk, 4 * H * dk] if nqk == 4 else [0, H * dk, 0, H * dk, 2 * H * dk]
    width = nqk * H * dk + H * dv
    qkv = (torch.randn(B * T, width, device=dev) * 0.7).bfloat16().requires_grad_()
    docs = make_docs(B, T).to(dev)
    power = 1.0 if kind == "offset_square" else 0.5
    tables = fused.attention_tables(docs)
    rs = row_scale_vector(docs, power).contiguous().view(-1)
    if kind == "offset_square":
        kpar = torch.full((H,), 0.7, device=dev, requires_grad=True)
    elif kind == "lower_degree_mix":
        kpar = torch.tensor([[0.1, 0.3, -0.2, 1.0]], device=dev).repeat(H, 1).requires_grad_()
    else:
        kpar = None
    y = fused.poly_attention(qkv, kpar, kind, dk, dv, H, cols, tables, rs)
    gy = torch.randn_like(y)
    y.backward(gy)
    torch.cuda.synchronize()
    assert lib().status() == 0
    qkv_ref = qkv.detach().double().requires_grad_()
    kpar_ref = kpar.detach().double().requires_grad_() if kpar is not None else None
    y_ref = dense_attention(kind, qkv_ref, cols, B, T, H, dk, dv, docs, power, kpar_ref)
    y_ref.backward(gy.double())
    assert rel(y.float(), y_ref) < 3e-2
    assert rel(qkv.grad.float(), qkv_ref.grad) < 3e-2
    if kpar is not None:
        assert rel(kpar.grad, kpar_ref.grad) < 3e-2


def test_rmsnorm_fwd_bwd_groups():
    torch.manual_seed(1)
    # one group at d = 1024 / 2048 / 4096 takes the single-pass kernel (two rows per step: odd counts)
    for groups, d, n in ((1, 512, 300), (4, 2048, 300), (1, 6144, 300), (1, 1024, 1301), (1, 2048, 777),
                         (1, 4096, 300)):
        x = torch.randn(n, d, device="cuda", requires_grad=True)
        w = (1 + 0.1 * torch.randn(d, device="cuda")).requires_grad_()
        y = fused.rms_norm(x, w, groups, 1e-6)
        gy = torch.randn(n, d, device="cuda").bfloat16()
        y.backward(gy)
        xr, wr = x.detach().double().requires_grad_(), w.detach().double().requires_grad_()
        xg = xr.unflatten(-1, (groups, -1))
        r = (xg.square().mean(-1, keepdim=True) + 1e-6).sqrt()
        yr = (xg / r).flatten(-2) * wr
        yr.backward(gy.double())
        assert rel(y.float(), yr) < 1e-2
        assert rel(x.grad, xr.grad) < 1e-2
        assert rel(w.grad, wr.grad) < 1e-2


def test_residual_norm_folds_dx_into_residual_grad_and_emits_bf16_copy():
    torch.manual_seed(2)
    for groups, d, n in ((1, 512, 200), (4, 2048, 200), (1, 6144, 200), (1, 2048, 1999), (1, 4096, 201)):
        x = torch.randn(n, d, device="cuda", requires_grad=True)
        w = (1 + 0.1 * torch.randn(d, device="cuda")).requires_grad_()
        xr, h = fused.residual_norm(x, w, groups, 1e-6, up_alpha=0.5)
        gres = torch.randn(n, d, device="cuda")
        gh = torch.randn(n, d, device="cuda").bfloat16()
        captured = {}

        def hook(g):
            captured["g"] = g
        x.register_hook(hook)
        torch.autograd.backward([xr, h], [gres.clone(), gh])
        xd, wd = x.detach().double().requires_grad_(), w.detach().double().requires_grad_()
        xg = xd.unflatten(-1, (groups, -1))
        r = (xg.square().mean(-1, keepdim=True) + 1e-6).sqrt()
        yr = (xg / r).flatten(-2) * wd
        (yr * gh.double()).sum().backward()
        expect = xd.grad + gres.double()
        assert rel(x.grad, expect) < 1e-2
        assert rel(w.grad, wd.grad) < 1e-2
        g16, alpha = captured["g"]._ttb_bf16
        assert alpha == 0.5 and g16.dtype == torch.bfloat16
        assert rel(g16.float(), 0.5 * expect) < 1e-2


def test_qkv_rope_gemm_matches_reference_rope():
    torch.manual_seed(5)
    from tensor_train_ing_b200.ops.block import rope_context
    B, T, H, dk = 2, 100, 2, 64
    docs = make_docs(B, T, pad=False).cuda()
    pos = doc_positions(docs)
    x = torch.randn(B * T, 256, device="cuda").bfloat16()
    w = (torch.randn(5 * H * dk, 256, device="cuda") / 16).bfloat16()
    rope = rope_context(pos.to(torch.int32).contiguous().view(-1), T, dk, 10000.0)
    out = lib().qkv_rope(x, w, 4 * H * dk, dk, rope["pos32"], rope["cos"], rope["sin"])
    raw = (x.float() @ w.float().t())
    cos, sin = rope_tables(pos, dk, 10000.0)
    qk = raw[:, :4 * H * dk].view(B, T, 4 * H, dk).transpose(1, 2)
    ref = apply_rope(qk, cos, sin).transpose(1, 2).reshape(B * T, -1)
    assert rel(out[:, :4 * H * dk].float(), ref) < 1e-2
    assert rel(out[:, 4 * H * dk:].float(), raw[:, 4 * H * dk:]) < 1e-2


def test_rope_roundtrip():
    torch.manual_seed(2)
    B, T, H, dk = 2, 100, 3, 64
    docs = make_docs(B, T, pad=False).cuda()
    pos = doc_positions(docs)
    qk = torch.randn(B * T, 2 * H * dk, device="cuda").bfloat16()
    buf = qk.clone()
    from tensor_train_ing_b200.models.attention import rope_inv_freq
    inv = rope_inv_freq(dk, 10000.0, "cuda")
    lib().rope_(buf, 2 * H * dk, dk, pos.to(torch.int32).contiguous().view(-1), inv, False)
    cos, sin = rope_tables(pos, dk, 10000.0)
    ref = apply_rope(qk.float().view(B, T, 2 * H, dk).transpose(1, 2), cos, sin).transpose(1, 2).reshape(B * T, -1)
    assert rel(buf.float(), ref) < 1e-2
    lib().rope_(buf, 2 * H * dk, dk, pos.to(torch.int32).contiguous().view(-1), inv, True)
    assert rel(buf.float(), qk.float()) < 2e-2


def test_linear_ce_matches_torch():
    torch.manual_seed(3)
    N, d, V, Vp = 700, 256, 1000, 1024
    from tensor_train_ing_b200.ops.weights import WeightGroup
    w = torch.nn.Parameter(torch.randn(Vp, d, device="cuda") * 0.05)
    x = torch.randn(N, d, device="cuda").bfloat16().requires_grad_()
    tgt = torch.randint(0, V, (N,), device="cuda")
    tgt[::7] = -100
    grp = WeightGroup([w])
    loss = fused.linear_cross_entropy(x, tgt, grp, V, alpha=0.5, chunk=256)
    loss.backward()
    xr = x.detach().double().requires_grad_()
    wr = w.detach().double().requires_grad_()
    logits = 0.5 * (xr @ wr[:V].t())
    lr = torch.nn.functional.cross_entropy(logits, tgt, ignore_index=-100, reduction="sum")
    lr.backward()
    assert abs(loss.item() - lr.item()) / abs(lr.item()) < 5e-3
    assert rel(x.grad.float(), xr.grad) < 3e-2
    assert rel(w.grad, wr.grad) < 3e-2
    assert w.grad[V:].abs().max().item() == 0.0


def test_embedding_deterministic_backward():
    torch.manual_seed(4)
    from tensor_train_ing_b200.ops.weights import WeightGroup
    W = torch.nn.Parameter(torch.randn(500, 128, device="cuda"))
    idx = torch.randint(0, 50, (4000,), device="cuda")
    grp = WeightGroup([W])
    x = fused.embedding(idx, grp)
    assert torch.equal(x, W.detach()[idx])
    g = torch.randn_like(x)
    x.backward(g)
    ref = torch.zeros_like(W).index_add_(0, idx, g)
    assert rel(W.grad, ref) < 1e-6
    first = W.grad.clone()
    W.grad = None
    fused.embedding(idx, grp).backward(g)
    assert torch.equal(W.grad, first)  # bitwise run-to-run determinism


def test_ce_backward_from_kept_logits_equals_recompute():
    """dlogits from the logits the forward kept == dlogits recomputed by the backward GEMM, and the
    two autograd paths give the same gradients."""
    torch.manual_seed(4)
    from tensor_train_ing_b200.ops._ext import lib
    from tensor_train_ing_b200.ops.weights import WeightGroup
    N, d, V, Vp = 300, 256, 1000, 1024
    x = torch.randn(N, d, device="cuda").bfloat16()
    w16 = (torch.randn(Vp, d, device="cuda") * 0.05).bfloat16()
    tgt = torch.randint(0, V, (N,), device="cuda")
    tgt[::5] = -100
    z = torch.full((N, Vp), float("nan"), device="cuda")
    _, lse = lib().ce_fwd(x, w16, V, 0.5, tgt, z)
    assert torch.isinf(z[:, V:]).all() and torch.isfinite(z[:, :V]).all()
    g = torch.full((1,), 0.25, device="cuda")
    d1 = torch.empty(N, Vp, device="cuda", dtype=torch.bfloat16)
    d2 = torch.empty_like(d1)
    lib().ce_bwd_logits(x, w16, V, 0.5, tgt, lse, g, d1)
    lib().ce_bwd_from_logits(z, 0.5, tgt, lse, g, d2)
    assert (d1.float() - d2.float()).abs().max().item() <= 1e-6
    grads = []
    for keep in (8 << 30, 0):
        fused.LinearCEFn.KEEP_LOGITS_BYTES = keep
        try:
            w = torch.nn.Parameter(w16.float())
            xg = x.clone().requires_grad_()
            loss = fused.linear_cross_entropy(xg, tgt, WeightGroup([w]), V, alpha=0.5, chunk=128)
            loss.backward()
            grads.append((loss.detach(), xg.grad, w.grad))
        finally:
            fused.LinearCEFn.KEEP_LOGITS_BYTES = 8 << 30
    for a, b in zip(grads[0], grads[1]):
        assert (a.float() - b.float()).abs().max().item() <= 1e-5 * max(1.0, b.float().abs().max().item())
    torch.cuda.synchronize()
    assert lib().status() == 0


def test_out_of_range_ids_and_targets_are_reported_and_skipped():
    """Token ids outside the embedding table and targets outside the vocabulary set the status word's
    bad-index code; the embedding writes zero rows (and drops their gradients) instead of reading
    outside the table, the loss of such a target row is zero, and later kernels run normally.  The
    table is a view with spare rows on both sides, so even a broken check would read mapped memory."""
    from tensor_train_ing_b200.ops._ext import check_status, lib
    V, d = 100, 64
    big = torch.randn(V + 2, d, device="cuda")
    W = big[1:V + 1]
    idx = torch.tensor([3, V, 7, -1, 5], device="cuda", dtype=torch.long)
    x = lib().embed_fwd(idx, W)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="index out of range"):
        check_status()
    assert torch.equal(x[[0, 2, 4]], W[[3, 7, 5]]) and not x[[1, 3]].any()
    dW = torch.zeros_like(W)
    spare = big[[0, V + 1]].clone()
    lib().embed_bwd(idx, torch.ones(5, d, device="cuda"), dW)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="index out of range"):
        check_status()
    assert torch.equal(dW[[3, 7, 5]], torch.ones(3, d, device="cuda")) and float(dW.abs().sum()) == 3 * d
    assert torch.equal(big[[0, V + 1]], spare)
    # a target past the vocabulary: no loss for its row, the others unchanged
    M, K, Vp = 256, 128, 128
    xs = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(Vp, K, device="cuda").bfloat16()
    tgt = torch.randint(0, V, (M,), device="cuda")
    loss_ok, _ = lib().ce_fwd(xs, w, V, 1.0, tgt)
    tgt_bad = tgt.clone()
    tgt_bad[10] = V + 3
    loss_bad, _ = lib().ce_fwd(xs, w, V, 1.0, tgt_bad)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="index out of range"):
        check_status()
    keep = torch.arange(M, device="cuda") != 10
    assert float(loss_bad[10]) == 0.0 and torch.equal(loss_bad[keep], loss_ok[keep])
    check_status()  # cleared: later launches report nothing
