"""The C entry point ``rmsnorm_bwd_noalloc`` (fixed device scratch, no allocation) against the
PyTorch binding ``rmsnorm_bwd`` of the same kernels, called through ctypes on the built library."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = 2


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
    _, rstd = _C.rmsnorm_fwd(x, w, G, 1e-6)
    return x, w, dy, dres, rstd


def _call(lib, x, w, dy, dres, rstd, dw, G, accumulate, dw_accumulate):
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.rmsnorm_bwd_noalloc(dy.data_ptr(), int(dy.dtype == torch.float32), x.data_ptr(), w.data_ptr(),
                                 rstd.data_ptr(), dres.data_ptr(), int(accumulate), dw.data_ptr(),
                                 int(dw_accumulate), x.shape[0], x.shape[1], G, stream)
    assert rc == 0, lib.rmsnorm_bwd_noalloc_last_error().decode()


@pytest.mark.parametrize("dy_dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_binding_twice_in_a_row(dy_dtype):
    from tensor_train_ing_b200 import _C
    lib = _cdll()
    # a larger call first, then a smaller one: the second reads only scratch rows it wrote itself
    for N, d, G, seed in ((3000, 512, 1, 0), (777, 384, 2, 1)):
        x, w, dy, dres, rstd = _case(N, d, G, dy_dtype, seed)
        dres_ref = dres.clone()
        dw_ref = _C.rmsnorm_bwd(dy, x, w, rstd, dres_ref, True, G)
        dres_c = dres.clone()
        dw_c = torch.full((d,), float("nan"), device="cuda")
        _call(lib, x, w, dy, dres_c, rstd, dw_c, G, accumulate=True, dw_accumulate=False)
        torch.cuda.synchronize()
        torch.testing.assert_close(dw_c, dw_ref, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(dres_c, dres_ref, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_sizes_beyond_scratch():
    lib = _cdll()
    cap = lib.rmsnorm_bwd_noalloc_max_scratch_floats()
    d = 4096
    N = 1 << 16
    assert lib.rmsnorm_bwd_noalloc_scratch_floats(N, d) > cap
    x = torch.zeros(1, 4, device="cuda")  # never read: the size check comes first
    rc = lib.rmsnorm_bwd_noalloc(x.data_ptr(), 1, x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 0,
                                 x.data_ptr(), 0, N, d, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
    assert b"scratch" in lib.rmsnorm_bwd_noalloc_last_error()
