"""Bitwise run-to-run determinism of the sm_100a kernels (B200).

Every reduction in these kernels has a fixed order (per-block partials summed in block order, no
floating-point atomics), so two runs on the same inputs must give identical bits.  Checked at op
level for the attention forward/backward (all kinds, several persistent-CTA counts), every GEMM
epilogue, the fused cross-entropy forward and both backward forms, RMSNorm backward on both launch
paths, the embedding backward, the norm-variant and spectral kernels and the optimizer kernels, and
at model level for a whole fused forward + backward.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

from tensor_train_ing_b200.ops import fused
from tensor_train_ing_b200.ops._ext import lib


def _same(a, b, what):
    if isinstance(a, (list, tuple)):
        for i, (x, y) in enumerate(zip(a, b)):
            _same(x, y, f"{what}[{i}]")
        return
    if a is None or (isinstance(a, torch.Tensor) and a.numel() == 0):
        return
    assert torch.equal(a, b), what


def twice(fn):
    torch.cuda.synchronize()
    first = fn()
    torch.cuda.synchronize()
    second = fn()
    torch.cuda.synchronize()
    return first, second


@pytest.mark.parametrize("kind", ["signed_product", "offset_square", "lower_degree_mix"])
def test_attention_forward_and_backward_are_bitwise_repeatable(kind):
    from test_kernels_gpu import make_docs
    torch.manual_seed(0)
    B, T, H, dk = 2, 384, 2, 128
    two = kind != "offset_square"
    cols = [0, H * dk, 2 * H * dk, 3 * H * dk, 4 * H * dk] if two else [0, H * dk, 0, H * dk, 2 * H * dk]
    qkv = (torch.randn(B * T, (5 if two else 3) * H * dk, device="cuda") * 0.3).bfloat16()
    docs = make_docs(B, T).cuda()
    tables = fused.attention_tables(docs)
    from tensor_train_ing_b200.models.attention import row_scale_vector
    rs = row_scale_vector(docs, 0.5).contiguous().view(-1)
    kpar = torch.randn(H, 4, device="cuda") * 0.3 if kind == "lower_degree_mix" else (
        torch.randn(H, device="cuda") * 0.2 if kind == "offset_square" else None)
    dy = torch.randn(B * T, H * dk, device="cuda").bfloat16()
    for limit in (0, 3):
        lib().attn_grid_limit(limit)
        try:
            def run():
                q = qkv.clone().requires_grad_(True)
                p = kpar.clone().requires_grad_(True) if kpar is not None else None
                y = fused.poly_attention(q, p, kind, dk, dk, H, cols, tables, rs)
                y.backward(dy)
                return [y.detach(), q.grad, p.grad if p is not None else None]
            a, b = twice(run)
            _same(a, b, f"attention {kind} limit {limit}")
        finally:
            lib().attn_grid_limit(0)


def test_gemm_epilogues_are_bitwise_repeatable():
    torch.manual_seed(1)
    M, K, N = 640, 512, 768
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    c = torch.randn(M, N, device="cuda")
    bias = torch.randn(N, device="cuda")

    def plain():
        out = torch.empty(M, N, device="cuda")
        lib().mm(a, b, out, c, 0.5, 1.0, bias, None)
        return out
    _same(*twice(plain), "mm alpha/beta/bias")
    wl = torch.randn(N, K, device="cuda").bfloat16()
    wr = torch.randn(N, K, device="cuda").bfloat16()

    def bilinear():
        h = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        l, r = torch.empty_like(h), torch.empty_like(h)
        lib().bilinear(a, wl, wr, None, None, 0, h, l, r)
        g = torch.randn(M, K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)).bfloat16()
        wd = wl.t().contiguous()
        dl, dr = torch.empty_like(l), torch.empty_like(r)
        lib().bilinear_grad(g, wd, l, r, dl, dr, 0)
        return [h, l, r, dl, dr]
    _same(*twice(bilinear), "bilinear / bilinear_grad")


def test_cross_entropy_forward_and_backward_are_bitwise_repeatable():
    torch.manual_seed(2)
    N, d, V, Vp = 900, 256, 1000, 1024
    x = torch.randn(N, d, device="cuda").bfloat16()
    w16 = (torch.randn(Vp, d, device="cuda") * 0.05).bfloat16()
    tgt = torch.randint(0, V, (N,), device="cuda")
    tgt[::9] = -100
    g = torch.full((1,), 0.25, device="cuda")

    def run():
        z = torch.empty(N, Vp, device="cuda")
        loss, lse = lib().ce_fwd(x, w16, V, 0.5, tgt, z)
        d1 = torch.empty(N, Vp, device="cuda", dtype=torch.bfloat16)
        d2 = torch.empty_like(d1)
        lib().ce_bwd_logits(x, w16, V, 0.5, tgt, lse, g, d1)
        lib().ce_bwd_from_logits(z, 0.5, tgt, lse, g, d2)
        return [loss, lse, z, d1, d2]
    _same(*twice(run), "cross entropy")


@pytest.mark.parametrize("d,groups", [(2048, 1), (768, 4)])
def test_rmsnorm_and_embedding_backward_are_bitwise_repeatable(d, groups):
    torch.manual_seed(3)
    N = 3000
    x = torch.randn(N, d, device="cuda")
    w = 1 + 0.1 * torch.randn(d, device="cuda")
    dy = torch.randn(N, d, device="cuda").bfloat16()
    _, rstd = lib().rmsnorm_fwd(x, w, groups, 1e-6)

    def run():
        dres = torch.zeros(N, d, device="cuda")
        dw = lib().rmsnorm_bwd(dy, x, w, rstd, dres, True, groups)
        return [dres, dw]
    _same(*twice(run), "rmsnorm backward")
    W = torch.randn(500, 256, device="cuda")
    idx = torch.randint(0, 64, (8000,), device="cuda")
    g = torch.randn(8000, 256, device="cuda")

    def emb():
        out = torch.zeros_like(W)
        lib().embed_bwd(idx, g, out)
        return out
    _same(*twice(emb), "embedding backward")


def test_norm_variant_spectral_and_optimizer_kernels_are_bitwise_repeatable():
    from tensor_train_ing_b200.models.normalization import SIGMA_FLOOR
    torch.manual_seed(4)
    N, d = 1000, 512
    x = torch.randn(N, d, device="cuda")
    w = 1 + 0.1 * torch.randn(d, device="cuda")
    w2 = torch.randn(d, device="cuda")
    dy = torch.randn(N, d, device="cuda")
    dr = torch.randn(N, device="cuda")

    def taper():
        y16, _, r, _ = lib().norm_variant_fwd(x, w, w2, 1, 0.4, 0.3, None, 1e-6, True, False, None, 1.0, True, False)
        return [y16, r] + list(lib().norm_variant_bwd(dy, x, w, w2, 1, 0.4, 0.3, None, 1e-6, 1.0, r, dr, None, False,
                                                      True, True))
    _same(*twice(taper), "taper norm")
    W = torch.randn(384, 512, device="cuda") * 0.05
    gamma = torch.full((1,), 1.3, device="cuda")
    u0 = torch.nn.functional.normalize(torch.randn(384, device="cuda"), dim=0)
    v0 = torch.nn.functional.normalize(torch.randn(512, device="cuda"), dim=0)
    G = torch.randn(384, 512, device="cuda")

    def spectral():
        u, v = u0.clone(), v0.clone()
        lib().spectral_power_step(W, u, v, SIGMA_FLOOR)
        out = torch.empty(384, 512, device="cuda", dtype=torch.bfloat16)
        sigma = lib().spectral_cast(W, gamma, u, v, SIGMA_FLOOR, out)
        return [u, v, sigma, out] + list(lib().spectral_grad(G, W, gamma, u, v, sigma, SIGMA_FLOOR))
    _same(*twice(spectral), "spectral")
    from tensor_train_ing_b200.optim import Muon

    def muon():
        p = torch.nn.Parameter(W.clone())
        opt = Muon([p], lr=0.02, weight_decay=0.1)
        for _ in range(2):
            p.grad = G.clone()
            opt.step(grad_scale=torch.tensor([0.7], device="cuda"))
        return [p.detach(), opt.state[p]["momentum_buffer"]]
    _same(*twice(muon), "muon")


@pytest.mark.parametrize("norm", ["pre_rms", "spectral_rms"])
def test_model_forward_backward_is_bitwise_repeatable(norm):
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    torch.manual_seed(5)
    cfg = ModelConfig(layers=2, d_model=256, heads=2, d_key=128, d_value=128, d_mlp=768, vocab_size=1000,
                      padded_vocab=1024, attention="signed_product", normalization=norm, loss_chunk_tokens=256)
    model = TensorLM(cfg).cuda()
    idx = torch.randint(0, 1000, (2, 300), device="cuda")
    docs = torch.zeros(2, 300, dtype=torch.long, device="cuda")
    docs[:, 120:] = 1
    tgt = torch.roll(idx, -1, 1)

    def run():
        model.zero_grad(set_to_none=True)
        _, loss, _ = model(idx, docs, tgt, reduction="sum")
        loss.backward()
        return [loss.detach()] + [p.grad.clone() for p in model.parameters() if p.grad is not None]
    _same(*twice(run), f"model {norm}")
