"""The C entry point ``rmsnorm_bwd_noalloc`` (fixed device scratch, no allocation), called through
ctypes on the built library, against an fp64 PyTorch RMSNorm backward and against the PyTorch
binding ``rmsnorm_bwd`` of the same kernels.

The cases cover both launch paths: the single-pass kernel the model takes for one group at
d = 1024 / 2048 / 4096, and the dx pass + weight-gradient pass used for other widths and groups.
Calls run back to back on one stream, larger before smaller, so a later call that read stale
scratch rows of an earlier one would show up as a mismatch.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = 2
EPS = 1e-6


def _cdll():
    from tensor_train_ing_b200 import _C
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p]
    lib.rmsnorm_bwd_noalloc_last_error.restype = ctypes.c_char_p
    lib.rmsnorm_bwd_noalloc_scratch_floats.restype = ctypes.c_longlong
    lib.rmsnorm_bwd_noalloc_scratch_floats.argtypes = [ctypes.c_int, ctypes.c_int]
    lib.rmsnorm_bwd_noalloc_max_scratch_floats.restype = ctypes.c_longlong
    return lib


def _case(N, d, G, dy_dtype, seed):
    from tensor_train_ing_b200 import _C
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(N, d, device="cuda", generator=g)
    w = 1 + 0.1 * torch.randn(d, device="cuda", generator=g)
    dy = torch.randn(N, d, device="cuda", generator=g).to(dy_dtype)
    dres = torch.randn(N, d, device="cuda", generator=g)
    _, rstd = _C.rmsnorm_fwd(x, w, G, EPS)
    return x, w, dy, dres, rstd


def _reference(x, w, dy, G):
    """dx and dw of sum(dy * rmsnorm(x) * w) with per-group statistics, by autograd in fp64."""
    xd = x.double().requires_grad_(True)
    wd = w.double().requires_grad_(True)
    N, d = x.shape
    xg = xd.view(N, G, d // G)
    r = (xg.pow(2).mean(-1, keepdim=True) + EPS).rsqrt()
    y = (xg * r).view(N, d) * wd
    dx, dw = torch.autograd.grad(y, (xd, wd), dy.double())
    return dx, dw


def _call(lib, x, w, dy, dres, rstd, dw, G, accumulate, dw_accumulate):
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.rmsnorm_bwd_noalloc(dy.data_ptr(), int(dy.dtype == torch.float32), x.data_ptr(), w.data_ptr(),
                                 rstd.data_ptr(), dres.data_ptr(), int(accumulate), dw.data_ptr(),
                                 int(dw_accumulate), x.shape[0], x.shape[1], G, stream)
    assert rc == 0, lib.rmsnorm_bwd_noalloc_last_error().decode()


# (N, d, G): single-pass path at d 4096 (at the documented 4096-row cap) and 2048, then the
# two-pass path at d 512 and 384 with two groups
CASES = [(4096, 4096, 1), (3000, 2048, 1), (3000, 512, 1), (777, 384, 2)]


@pytest.mark.parametrize("dy_dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_fp64_and_binding_twice_in_a_row(dy_dtype):
    from tensor_train_ing_b200 import _C
    lib = _cdll()
    cap = lib.rmsnorm_bwd_noalloc_max_scratch_floats()
    for rep in range(2):
        for k, (N, d, G) in enumerate(CASES):
            if lib.rmsnorm_bwd_noalloc_scratch_floats(N, d) > cap:
                continue  # a GPU with more SMs than the 148 the stated row caps assume
            x, w, dy, dres, rstd = _case(N, d, G, dy_dtype, seed=10 * rep + k)
            dx64, dw64 = _reference(x, w, dy, G)
            # binding (allocates its partials through torch): dres accumulates, dw is written
            dres_ref = dres.clone()
            dw_ref = _C.rmsnorm_bwd(dy, x, w, rstd, dres_ref, True, G)
            # entry point: dres accumulates, dw is written over a NaN fill
            dres_c = dres.clone()
            dw_c = torch.full((d,), float("nan"), device="cuda")
            _call(lib, x, w, dy, dres_c, rstd, dw_c, G, accumulate=True, dw_accumulate=False)
            torch.cuda.synchronize()
            # the same kernels in the same order: the binding's results exactly
            torch.testing.assert_close(dw_c, dw_ref, rtol=0, atol=0)
            torch.testing.assert_close(dres_c, dres_ref, rtol=0, atol=0)
            # against fp64: fp32 row reductions over d and fp32 column sums over N rows
            torch.testing.assert_close(dres_c.double(), dres.double() + dx64, rtol=1e-4, atol=1e-4)
            torch.testing.assert_close(dw_c.double(), dw64, rtol=1e-4, atol=1e-3 * (N / 1000) ** 0.5)


def test_noalloc_overwrite_and_accumulate_modes():
    """accumulate=0 overwrites the residual gradient; dw_accumulate=1 adds to a pre-filled dw."""
    lib = _cdll()
    for N, d, G in ((2048, 2048, 1), (600, 768, 4)):
        x, w, dy, dres, rstd = _case(N, d, G, torch.bfloat16, seed=N)
        dx64, dw64 = _reference(x, w, dy, G)
        prior = torch.linspace(-1, 1, d, device="cuda")
        dres_c = torch.full_like(dres, float("nan"))
        dw_c = prior.clone()
        _call(lib, x, w, dy, dres_c, rstd, dw_c, G, accumulate=False, dw_accumulate=True)
        torch.cuda.synchronize()
        torch.testing.assert_close(dres_c.double(), dx64, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(dw_c.double(), prior.double() + dw64, rtol=1e-4, atol=2e-3)


def test_noalloc_rejects_sizes_beyond_scratch():
    lib = _cdll()
    cap = lib.rmsnorm_bwd_noalloc_max_scratch_floats()
    d = 8192
    N = 8
    # grow N until the partial rows times d exceed the array (they stop growing at 4 rows per SM)
    while lib.rmsnorm_bwd_noalloc_scratch_floats(N, d) <= cap and N < (1 << 24):
        N *= 2
    if lib.rmsnorm_bwd_noalloc_scratch_floats(N, d) <= cap:
        pytest.skip("this GPU has too few SMs for any call to exceed the scratch array")
    x = torch.zeros(1, 4, device="cuda")  # never read: the size check comes first
    rc = lib.rmsnorm_bwd_noalloc(x.data_ptr(), 1, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 0,
                                 x.data_ptr(), 0, N, d, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
    assert b"scratch" in lib.rmsnorm_bwd_noalloc_last_error()
