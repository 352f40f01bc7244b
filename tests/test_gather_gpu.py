"""The all-gather fused into the CTA-pair GEMM (csrc/gemm/gather.cuh) on one GPU.

The ranks' row shards are separate local buffers here (their addresses stand in for the peer
mappings; the two-GPU worker tests/dist_workers/sharded_params_gpu.py reads real peers), so every
part of the kernel runs: chunk claims, copies, per-slab done words, the producer's waits, the
counter reset, and repeated gathers of one buffer (done words at one, two and three times the chunks per slab).  Each gathered GEMM
must equal the same GEMM on the full weight bit for bit (same kernel arithmetic, same operand
values) and leave the weight in its staging buffer.
"""
import pytest
import torch

from tensor_train_ing_b200.parallel.gather import GatheredWeight, GatherWindow, chunks_per_slab, row_cuts

pytestmark = pytest.mark.gpu


def _lib():
    from tensor_train_ing_b200.ops._ext import lib
    return lib()


class _Shards:
    """A weight split into per-rank row shards held in separate buffers, with its done words."""

    def __init__(self, w: torch.Tensor, world: int):
        self.cuts = row_cuts(w.shape[0], world)
        self.shards = [w[a:b].clone() for a, b in zip(self.cuts, self.cuts[1:])]
        self.done = torch.zeros(w.shape[0] // 64, dtype=torch.int32, device=w.device)
        self.uses = 0
        # an empty shard still needs an aligned address: any valid one (it is never read)
        self.ptrs = [s.data_ptr() if s.numel() else w.data_ptr() for s in self.shards]

    def spec(self):
        self.uses += 1
        return (self.ptrs, self.cuts, self.done, self.uses)

    def update(self, w):
        for s, (a, b) in zip(self.shards, zip(self.cuts, self.cuts[1:])):
            s.copy_(w[a:b])


@pytest.mark.parametrize("M,N,K,world", [(1024, 1280, 512, 3), (512, 768, 256, 8), (200, 512, 256, 2),
                                         (2048, 2048, 1024, 5)])
def test_gathered_linear_equals_the_plain_gemm(M, N, K, world):
    torch.manual_seed(M + N + world)
    x = torch.randn(M, K, device="cuda").bfloat16()
    shards = None
    for rep in range(3):  # the same staging buffer and done words, new weights each time
        w = torch.randn(N, K, device="cuda").bfloat16()
        if shards is None:
            shards = _Shards(w, world)
        else:
            shards.update(w)
        staging = torch.full_like(w, float("nan"))
        got = torch.empty(M, N, device="cuda", dtype=torch.float32)
        _lib().mm(x, staging.t(), got, None, 1.0, 0.0, None, None, 0, [shards.spec()])
        want = torch.empty_like(got)
        _lib().mm(x, w.t(), want)
        torch.cuda.synchronize()
        assert _lib().status() == 0
        assert torch.equal(staging, w), f"staging differs from the weight (call {rep})"
        assert torch.equal(got, want), f"gathered GEMM differs (call {rep})"
        ref = x.float() @ w.float().t()
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-2)
        assert int(shards.done.min()) == int(shards.done.max()) == chunks_per_slab(K) * (rep + 1)


def test_gathered_qkv_rope_and_bilinear_equal_the_plain_kernels():
    torch.manual_seed(0)
    M, K, H, dk, F = 1024, 512, 4, 64, 768
    x = torch.randn(M, K, device="cuda").bfloat16()
    # QKV with the rotary epilogue
    w = (torch.randn(5 * H * dk, K, device="cuda") / K ** 0.5).bfloat16()
    pos = torch.arange(M, device="cuda", dtype=torch.int32) % 256
    inv = 1.0 / (10000 ** (torch.arange(0, dk, 2, device="cuda").float() / dk))
    ang = torch.arange(256, device="cuda").float()[:, None] * inv[None]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    sh = _Shards(w, 4)
    staging = torch.empty_like(w)
    got = _lib().qkv_rope(x, staging, 4 * H * dk, dk, pos, cos, sin, None, [sh.spec()])
    want = _lib().qkv_rope(x, w, 4 * H * dk, dk, pos, cos, sin)
    # bilinear: two staged operands, slabs interleaved
    wl = (torch.randn(F, K, device="cuda") / K ** 0.5).bfloat16()
    wr = (torch.randn(F, K, device="cuda") / K ** 0.5).bfloat16()
    sl, sr = _Shards(wl, 3), _Shards(wr, 3)
    stl, str_ = torch.empty_like(wl), torch.empty_like(wr)
    outs = [torch.empty(M, F, device="cuda", dtype=torch.bfloat16) for _ in range(6)]
    _lib().bilinear(x, stl, str_, None, None, 0, outs[0], outs[1], outs[2], [sl.spec(), sr.spec()])
    _lib().bilinear(x, wl, wr, None, None, 0, outs[3], outs[4], outs[5])
    torch.cuda.synchronize()
    assert _lib().status() == 0
    assert torch.equal(staging, w) and torch.equal(got, want)
    assert torch.equal(stl, wl) and torch.equal(str_, wr)
    for a, b in zip(outs[:3], outs[3:]):
        assert torch.equal(a, b)


def test_gather_rows_alone_and_the_window():
    """The copy without a GEMM (the path of consumers that are not CTA-pair GEMMs) and the window's
    residency: a second request of a resident group gathers nothing, an invalidated one again."""
    torch.manual_seed(1)
    w = torch.randn(640, 256, device="cuda").bfloat16()
    sh = _Shards(w, 2)
    window = GatherWindow("cuda", 2, w.numel())
    gw = GatheredWeight(window, 640, 256, sh.cuts, sh.ptrs)
    view = gw.resident()
    torch.cuda.synchronize()
    assert _lib().status() == 0 and torch.equal(view, w) and window.gathers == 1
    assert gw.resident().data_ptr() == view.data_ptr() and window.gathers == 1
    w2 = torch.randn_like(w)
    sh.update(w2)
    window.invalidate()
    view = gw.resident()
    torch.cuda.synchronize()
    assert torch.equal(view, w2) and window.gathers == 2 and int(gw.done.min()) == 2 * chunks_per_slab(256)
