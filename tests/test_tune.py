"""The kernel tuner's host side: shape parsing, the results table and installing it (CPU)."""
import json

import pytest

from tensor_train_ing_b200 import tune
from tensor_train_ing_b200.ops import fused


def test_shape_parsing():
    assert tune.parse_shape("16384x2048x8192") == (16384, 2048, 8192)
    for bad in ("16x16", "0x8x8", "axbxc"):
        with pytest.raises(ValueError):
            tune.parse_shape(bad)


def test_best_choices_merge_into_one_table_and_install(tmp_path):
    path = tmp_path / "tuning.json"
    tune.merge_best(path, "gemm", [{"shape": "512x1024x256", "tile_n": 128, "ms": 0.1}], {})
    tune.merge_best(path, "gemm", [{"shape": "8192x8192x8192", "tile_n": 256, "ms": 2.0}], {})
    tune.merge_best(path, "attention", [{"grid_limit": 132, "ms": 1.0}], {"batch": 8})
    tune.merge_best(path, "step", [{"micro_batch": 8, "loss_chunk_tokens": 8192, "ms_per_step": 9.0}],
                    {"preset": "bench_1b"})
    table = json.loads(path.read_text())
    assert table["gemm_tiles"] == {"512x1024x256": 128, "8192x8192x8192": 256}
    assert table["attention_grid_limit"] == 132 and table["step_advice"][0]["best"]["micro_batch"] == 8
    try:
        assert tune.apply(path) == {"gemm_tiles": 2, "attention_grid_limit": 132}
        assert fused.GEMM_TILES == {(512, 1024, 256): 128, (8192, 8192, 8192): 256}
    finally:
        fused.GEMM_TILES.clear()


def test_invalid_tables_are_refused():
    with pytest.raises(ValueError):
        tune.apply({"gemm_tiles": {"64x64x64": 192}})
    with pytest.raises(ValueError):
        tune.apply({"attention_grid_limit": -1})
    assert fused.GEMM_TILES == {}
