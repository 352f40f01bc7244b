"""The day-one canary on a B200: numerics checks pass and the throughput gate decides."""
import json

import pytest

from tensor_train_ing_b200.runbook import canary

pytestmark = pytest.mark.gpu


def test_canary_numerics_and_short_throughput_gate(tmp_path):
    checks = canary.numerics_checks()
    assert {c["check"] for c in checks} == {"gemm", "rmsnorm", "cross_entropy", "polynomial_attention_fwd_bwd"}
    assert all(c["ok"] for c in checks), checks
    report = canary.run_canary(tmp_path / "canary", preset="screen_100m", context=512, rows_per_rank=4,
                               micro_batch=2, steps=4, warmup_steps=1, min_tokens_per_second=1.0)
    assert report["status"] == "passed" and report["throughput_gate"]["status"] == "passed"
    assert report["tokens_per_second"] > 0 and len(report["steps"]) == 4
    assert json.loads((tmp_path / "canary" / "result.json").read_text())["status"] == "passed"
