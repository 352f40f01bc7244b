"""tcgen05 GEMM family vs a plain fp32 PyTorch reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from tensor_train_ing_b200.ops._ext import lib
    return lib()


def _ref(a, b):
    return a.float() @ b.float()


def _rel(x, y):
    return ((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (300, 200, 96), (1000, 1536, 1000),
                                   (129, 130, 136), (4096, 2048, 2048)])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
def test_mm_layouts(M, N, K, a_t, b_t):
    torch.manual_seed(0)
    dev = "cuda"
    a = (torch.randn(K, M, device=dev).t() if a_t else torch.randn(M, K, device=dev)).bfloat16()
    b = (torch.randn(N, K, device=dev).t() if b_t else torch.randn(K, N, device=dev)).bfloat16()
    if a_t:
        a = a.t().contiguous().t()
    if b_t:
        b = b.t().contiguous().t()
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    lds = [K, N if not b_t else K] + ([M] if a_t else []) + ([N] if not b_t else [])
    if any(ld % 8 for ld in lds):
        with pytest.raises(ValueError):  # TMA needs 16-byte row strides: rejected loudly
            _C().mm(a, b, out)
        return
    _C().mm(a, b, out)
    torch.cuda.synchronize()
    assert _C().status() == 0
    assert _rel(out, _ref(a, b)) < 1e-2


def test_mm_fp32_accumulate_bias_alpha():
    torch.manual_seed(1)
    M, N, K = 512, 384, 320
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(K, N, device="cuda").bfloat16()
    c = torch.randn(M, N, device="cuda")
    bias = torch.randn(N, device="cuda")
    out = c.clone()
    _C().mm(a, b, out, c=out, alpha=0.5, beta=1.0, bias=bias)
    ref = 0.5 * (_ref(a, b) + bias) + c
    assert _rel(out, ref) < 1e-5 * 100


def test_bilinear_and_grad():
    torch.manual_seed(2)
    M, K, N = 640, 256, 384
    x = torch.randn(M, K, device="cuda").bfloat16()
    wl = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    wr = (torch.randn(N, K, device="cuda") / K ** 0.5).bfloat16()
    h = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    lo, ro = torch.empty_like(h), torch.empty_like(h)
    _C().bilinear(x, wl, wr, None, None, 0, h, lo, ro)
    l_ref = (x.float() @ wl.float().t())
    r_ref = (x.float() @ wr.float().t())
    assert _rel(lo, l_ref) < 1e-2 and _rel(ro, r_ref) < 1e-2
    assert _rel(h, l_ref * r_ref) < 2e-2
    # backward: dH = dy @ wd, dl = dH*r, dr = dH*l
    D = 192
    wd = (torch.randn(D, N, device="cuda") / N ** 0.5).bfloat16()
    dy = torch.randn(M, D, device="cuda").bfloat16()
    dl, dr = torch.empty_like(h), torch.empty_like(h)
    _C().bilinear_grad(dy, wd, lo, ro, dl, dr, 0)
    dh = dy.float() @ wd.float()
    assert _rel(dl, dh * ro.float()) < 2e-2 and _rel(dr, dh * lo.float()) < 2e-2
    torch.cuda.synchronize()
    assert _C().status() == 0


@pytest.mark.parametrize("M,N,K1,K2", [(512, 256, 128, 192), (4096, 2048, 1024, 1024), (300, 200, 64, 96)])
@pytest.mark.parametrize("b_t", [False, True])
def test_mm_concatenated_contraction(M, N, K1, K2, b_t):
    """a @ cat(b1, b2) in one pass (the bilinear MLP's dx = [dl | dr] @ [L; R])."""
    torch.manual_seed(3)
    a = torch.randn(M, K1 + K2, device="cuda").bfloat16()
    mk = (lambda k: torch.randn(N, k, device="cuda").bfloat16().t()) if b_t else \
        (lambda k: torch.randn(k, N, device="cuda").bfloat16())
    b1, b2 = mk(K1), mk(K2)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    _C().mm(a, b1, out, b2=b2)
    torch.cuda.synchronize()
    assert _C().status() == 0
    assert _rel(out, _ref(a, torch.cat([b1, b2], 0))) < 1e-2
    with pytest.raises(RuntimeError):  # the split must fall on a 64-wide k-block
        _C().mm(a[:, 1:], b1[1:], out, b2=b2)


def test_bilinear_grad_strided_outputs():
    """dl, dr written as the two halves of one [M, 2N] buffer."""
    torch.manual_seed(4)
    M, N, D = 640, 384, 256
    lo = torch.randn(M, N, device="cuda").bfloat16()
    ro = torch.randn(M, N, device="cuda").bfloat16()
    wd = (torch.randn(D, N, device="cuda") / N ** 0.5).bfloat16()
    dy = torch.randn(M, D, device="cuda").bfloat16()
    dlr = torch.full((M, 2 * N), float("nan"), device="cuda", dtype=torch.bfloat16)
    _C().bilinear_grad(dy, wd, lo, ro, dlr[:, :N], dlr[:, N:], 0)
    dh = dy.float() @ wd.float()
    assert _rel(dlr[:, :N], dh * ro.float()) < 2e-2 and _rel(dlr[:, N:], dh * lo.float()) < 2e-2
    torch.cuda.synchronize()
    assert _C().status() == 0


@pytest.mark.parametrize("M,N,D", [(300, 200, 136), (256, 520, 64)])
@pytest.mark.parametrize("mode", [0, 1])
def test_bilinear_grad_ragged_edges(M, N, D, mode):
    """Column counts that end inside a 32-column chunk and rows that end inside a tile."""
    torch.manual_seed(5)
    lo = torch.randn(M, N, device="cuda").bfloat16()
    ro = torch.randn(M, N, device="cuda").bfloat16()
    wd = (torch.randn(D, N, device="cuda") / N ** 0.5).bfloat16()
    dy = torch.randn(M, D, device="cuda").bfloat16()
    dl, dr = torch.empty_like(lo), torch.empty_like(lo)
    _C().bilinear_grad(dy, wd, lo, ro, dl, dr, mode)
    dh = (dy.float() @ wd.float()).bfloat16().float()
    l, r = lo.float(), ro.float()
    if mode == 0:
        want_l, want_r = dh * r, dh * l
    else:
        sg = torch.sigmoid(l)
        want_l, want_r = dh * r * sg * (1 + l * (1 - sg)), dh * l * sg
    assert _rel(dl, want_l) < 2e-2 and _rel(dr, want_r) < 2e-2
    torch.cuda.synchronize()
    assert _C().status() == 0
