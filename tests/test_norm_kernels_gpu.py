"""Norm-variant and spectral-linear kernels against fp64 PyTorch references of the same ops (B200).

Tolerances (fixed before the kernels were written): fp32 outputs within rtol 1e-4 / atol 1e-5 of
fp64 (fp32 row reductions over d <= 2048); bf16 outputs within one bf16 ulp (rtol 8e-3); the power
iteration's vectors within 1e-5.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

LAGGED, TAPER, RMS = 0, 1, 2


def _lib():
    from tensor_train_ing_b200.ops._ext import lib
    return lib()


def _data(N, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(N, d, device="cuda", generator=g) * 1.7
    w = 1 + 0.2 * torch.randn(d, device="cuda", generator=g)
    w2 = 0.5 + 0.2 * torch.randn(d, device="cuda", generator=g)
    dy = torch.randn(N, d, device="cuda", generator=g)
    return x, w, w2, dy


@pytest.mark.parametrize("dy_dtype", [torch.float32, torch.bfloat16])
def test_lagged_variant_forward_backward(dy_dtype):
    x, w, _, dy = _data(300, 512, 0)
    dy = dy.to(dy_dtype)
    mean_sq = torch.tensor(2.7, dtype=torch.float64, device="cuda")
    scale = (mean_sq + 1e-6).sqrt().reciprocal().float().reshape(1)
    y16, _, _, msq = _lib().norm_variant_fwd(x, w, None, LAGGED, 0.0, 0.0, scale, 1e-6, True, False, None, 1.0,
                                             False, True)
    xd, wd = x.double().requires_grad_(True), w.double().requires_grad_(True)
    ref = xd / (mean_sq + 1e-6).sqrt() * wd
    torch.testing.assert_close(y16.double(), ref.detach(), rtol=8e-3, atol=1e-3)
    torch.testing.assert_close(msq.double(), x.double().pow(2).mean(-1), rtol=1e-5, atol=1e-6)
    dxr, dwr = torch.autograd.grad(ref, (xd, wd), dy.double())
    dx, dw, _ = _lib().norm_variant_bwd(dy, x, w, None, LAGGED, 0.0, 0.0, scale, 1e-6, 1.0, None, None, None, False,
                                        True, False)
    torch.testing.assert_close(dx.double(), dxr, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dw.double(), dwr, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("g", [1.0, 0.35, 0.0])
def test_taper_variant_with_anchor_gradient(g):
    x, w, w2, dy = _data(257, 768, 1)
    c, eps = 0.8, 1e-6
    b = (1 - g) * c
    y16, _, r, _ = _lib().norm_variant_fwd(x, w, w2, TAPER, g, b, None, eps, True, False, None, 1.0, True, False)
    xd, wd, w2d = (t.double().requires_grad_(True) for t in (x, w, w2))
    rd = (xd.pow(2).mean(-1, keepdim=True) + eps).sqrt()
    ref = g * (xd / rd * wd) + b * xd * w2d
    torch.testing.assert_close(r.double(), rd.squeeze(-1).detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(y16.double(), ref.detach(), rtol=8e-3, atol=1e-3)
    dr = torch.linspace(-0.5, 0.5, x.shape[0], device="cuda")  # gradient arriving through r (the anchor)
    dxr, dwr, dw2r = torch.autograd.grad((ref, rd.squeeze(-1)), (xd, wd, w2d), (dy.double(), dr.double()))
    dx, dw, dw2 = _lib().norm_variant_bwd(dy, x, w, w2 if b else None, TAPER, g, b, None, eps, 1.0, r, dr, None,
                                          False, g != 0.0, b != 0.0)
    torch.testing.assert_close(dx.double(), dxr, rtol=1e-4, atol=1e-5)
    if g:
        torch.testing.assert_close(dw.double(), dwr, rtol=1e-4, atol=1e-4)
    if b:
        torch.testing.assert_close(dw2.double(), dw2r, rtol=1e-4, atol=1e-4)


def test_output_rms_variant_adds_into_the_stream():
    z, w, _, dy = _data(200, 1024, 2)
    resid = torch.randn_like(z)
    alpha, eps = 0.7, 1e-6
    _, y32, r, _ = _lib().norm_variant_fwd(z, w, None, RMS, 0.0, 0.0, None, eps, False, True, resid, alpha, True,
                                           False)
    zd, wd = z.double().requires_grad_(True), w.double().requires_grad_(True)
    ref = resid.double() + alpha * (zd / (zd.pow(2).mean(-1, keepdim=True) + eps).sqrt() * wd)
    torch.testing.assert_close(y32.double(), ref.detach(), rtol=1e-4, atol=1e-5)
    dzr, dwr = torch.autograd.grad(ref, (zd, wd), dy.double())
    accum = torch.randn_like(z)
    dz, dw, _ = _lib().norm_variant_bwd(dy, z, w, None, RMS, 0.0, 0.0, None, eps, alpha, r, None, accum.clone(), True,
                                        True, False)
    torch.testing.assert_close(dz.double(), accum.double() + dzr, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dw.double(), dwr, rtol=1e-4, atol=1e-4)


def test_spectral_power_step_cast_and_grad():
    from tensor_train_ing_b200.models.normalization import SIGMA_FLOOR, SpectralLinear
    torch.manual_seed(0)
    lin = SpectralLinear(384, 300).cuda()
    torch.nn.init.normal_(lin.weight, std=0.05)
    u0, v0 = lin.u.clone(), lin.v.clone()
    w64 = lin.weight.detach().double()
    vt = w64.t() @ u0.double()
    vt = vt / vt.norm()
    ut = w64 @ vt
    ut = ut / ut.norm()
    _lib().spectral_power_step(lin.weight.detach(), lin.u, lin.v, SIGMA_FLOOR)
    torch.testing.assert_close(lin.v.double(), vt, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lin.u.double(), ut, rtol=1e-5, atol=1e-6)
    with torch.no_grad():
        lin.gamma.fill_(1.9)
    out = torch.empty(300, 384, device="cuda", dtype=torch.bfloat16)
    sigma = _lib().spectral_cast(lin.weight.detach(), lin.gamma.detach(), lin.u, lin.v, SIGMA_FLOOR, out)
    wd = lin.weight.detach().double().requires_grad_(True)
    gd = lin.gamma.detach().double().requires_grad_(True)
    sig = lin.u.double() @ wd @ lin.v.double()
    eff = gd * wd / sig.abs().clamp_min(SIGMA_FLOOR)
    torch.testing.assert_close(sigma.double(), sig.detach().reshape(1), rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(out.double(), eff.detach(), rtol=8e-3, atol=1e-4)
    G = torch.randn(300, 384, device="cuda")
    dwr, dgr = torch.autograd.grad(eff, (wd, gd), G.double())
    dw, dg = _lib().spectral_grad(G, lin.weight.detach(), lin.gamma.detach(), lin.u, lin.v, sigma, SIGMA_FLOOR)
    torch.testing.assert_close(dw.double(), dwr, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dg.double(), dgr, rtol=1e-4, atol=1e-6)


def test_spectral_step_on_cuda_matches_the_cpu_iteration():
    from tensor_train_ing_b200.models.normalization import SpectralLinear, spectral_step
    torch.manual_seed(1)
    cpu = SpectralLinear(256, 192)
    torch.nn.init.normal_(cpu.weight, std=0.1)
    gpu = SpectralLinear(256, 192).cuda()
    gpu.load_state_dict(cpu.state_dict())
    for _ in range(3):
        spectral_step(cpu)
        spectral_step(gpu)
    torch.testing.assert_close(gpu.u.cpu(), cpu.u, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(gpu.v.cpu(), cpu.v, rtol=1e-5, atol=1e-6)
