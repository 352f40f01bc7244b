"""Tuner sweeps on the B200: every GEMM tile width gives the same bits (and matches an fp32
reference), the attention grid limits all run, and an installed table reaches the GEMM wrapper."""
import pytest
import torch

from tensor_train_ing_b200 import tune
from tensor_train_ing_b200.ops import fused

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(512, 1024, 256), (1000, 384, 320)])
def test_gemm_tiles_agree(shape):
    rows = tune.sweep_gemm(shape, reps=2)  # raises if the two tiles differ in any bit
    assert {r["tile_n"] for r in rows} == {128, 256} and all(r["ms"] > 0 for r in rows)
    M, N, K = shape
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(N, K, device="cuda").bfloat16()
    want = a.float() @ b.float().t()
    for tile in (128, 256):
        fused.GEMM_TILES[(M, N, K)] = tile
        try:
            got = fused._mm(a, b.t(), torch.empty(M, N, device="cuda"))
        finally:
            fused.GEMM_TILES.clear()
        torch.testing.assert_close(got, want, rtol=2e-3, atol=2e-3)


def test_attention_grid_sweep_runs_every_limit():
    rows = tune.sweep_attention(batch=2, context=512, heads=2, head_dim=128, doc_len=200, grids=(0, 8, 3), reps=2)
    assert sorted(r["grid_limit"] for r in rows) == [0, 3, 8] and all(r["ms"] > 0 for r in rows)
