"""Coordinate check and the per-update profiler on CPU (their GPU use is the same code with CUDA
activity enabled)."""
import json

import pytest
import torch

from tensor_train_ing_b200.coordcheck import run, run_depth
from tensor_train_ing_b200.profiling import KernelProfile


def test_width_coordinate_check_reports_every_probe_and_slopes():
    out = run(widths=(32, 64), layers=2, head_dim=16, steps=2, batch=2, context=16, vocab=64, device="cpu")
    assert out["widths"] == [32, 64] and set(out["rows"]) == {32, 64}
    keys = set(out["rows"][32])
    assert {"logits", "resid0", "resid1", "attn1", "mlp1"} <= keys
    for row in out["rows"].values():
        for stats in row.values():
            assert all(v >= 0 and v == v for v in stats.values())  # finite, nonnegative RMS values
    assert set(out["loglog_slopes"]) == {f"{k}.{f}" for k in keys for f in ("init", "delta")}


def test_depth_coordinate_check():
    out = run_depth(depths=(1, 2), width=32, head_dim=16, steps=1, batch=2, context=16, vocab=64, device="cpu")
    assert out["depths"] == [1, 2] and "resid_last.delta" in out["loglog_slopes"]


def test_kernel_profile_captures_after_warmup_and_writes_a_trace(tmp_path):
    prof = KernelProfile(warmup_steps=1, trace_dir=tmp_path / "trace", trace_steps=2, cuda=False)
    x = torch.randn(64, 64)
    for step in range(4):
        prof.start_step(step)
        with prof.region("matmul"):
            y = x @ x
        prof.finish_step()
    prof.close()
    assert prof.steps == [1, 2]  # step 0 was warm-up; two steps captured
    rep = prof.report()
    assert rep["captured_steps"] == [1, 2] and "kernels" in rep
    traces = list((tmp_path / "trace").glob("trace-steps-1-2.json"))
    assert len(traces) == 1 and json.loads(traces[0].read_text())
    assert y.shape == (64, 64)


def test_launch_count_of_the_rmsnorm_backward_follows_its_kernel_path():
    from tensor_train_ing_b200.ops._ext import KERNELS_PER_CALL
    count = KERNELS_PER_CALL["rmsnorm_bwd"]
    for d, groups, kernels in ((2048, 1, 2), (1024, 1, 2), (4096, 1, 2), (6144, 1, 3), (2048, 4, 3), (512, 1, 3)):
        x = torch.empty(3, d)
        assert count(x, x, None, None, x, True, groups) == kernels


def test_attention_scaling_fit_recovers_fixed_and_per_block_costs(monkeypatch):
    """kernel_bench attn_scale: with timings exactly fixed + per_block * blocks, the fit returns them."""
    from tensor_train_ing_b200 import kernel_bench as kb

    class FakeLib:
        def poly_fwd(self, *a):
            return ("fwd", a[9], a[10])

        def poly_bwd(self, *a):
            return ("bwd", a[11], a[12])

    blocks = {}

    def fake_inputs(b, t):
        nq = t // 128
        blocks[(b, t)] = b * kb.H * sum(2 * (q + 1) for q in range(nq))
        return {"pos32": 0, "doc32": 0, "doc_end32": 0}, 0, 0, 0, 0, 0, {"cos": 0, "sin": 0}

    def fake_time(fn, reps=10):
        kind, b, t = fn()
        fixed, per = (60.0, 0.006) if kind == "fwd" else (240.0, 0.024)
        return fixed + per * blocks[(b, t)]

    monkeypatch.setattr(kb, "_lib", lambda: FakeLib())
    monkeypatch.setattr(kb, "_attn_inputs", fake_inputs)
    monkeypatch.setattr(kb, "_event_time", fake_time)
    import tensor_train_ing_b200.ops._ext as ext
    monkeypatch.setattr(ext, "check_status", lambda: None)
    out = kb.attn_scaling(rope=True)
    assert out["fit"]["fwd"] == {"fixed_us": pytest.approx(60.0, abs=0.2), "ns_per_block": pytest.approx(6.0, abs=0.01)}
    assert out["fit"]["bwd"] == {"fixed_us": pytest.approx(240.0, abs=0.2), "ns_per_block": pytest.approx(24.0, abs=0.01)}
