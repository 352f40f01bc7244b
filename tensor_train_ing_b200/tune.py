"""Sweeps of the runtime choices the sm_100a kernels expose, measured on the GPU at hand.  The
counterpart of the reference's Triton tile / stage / warp sweep (tnlm/kernels/tune.py:20-62): the
tile shapes of these kernels are fixed where they are compiled, so what remains to choose at run
time is swept here.

* ``attention``: the grid of the persistent polynomial-attention kernels (how many CTAs run at
  once; the rest of the tiles are handed out by a device counter), forward and backward timed
  together at a batch / context / heads / head dim / document length;
* ``gemm``: the output tile of the linear GEMM per shape: 128 (one CTA per 128 x 128 tile, six K
  stages) or 256 (a CTA pair on a 256 x 256 tile with ``cta_group::2`` MMAs, four stages);
* ``step``: micro-batch size and fused cross-entropy chunk of a whole training step (``TrainEngine``)
  at a benchmark shape (``bench_1b`` and the like).

Each timing is CUDA events on the current stream after three warm-up calls, each timed call after
a 256 MB write that flushes L2.  A sweep prints every candidate, fastest first.  ``--write PATH``
merges the best choices into a JSON file; ``apply(PATH)`` (or ``TTB_TUNING=PATH`` when the kernel
library loads) installs the attention grid and the per-shape GEMM tiles in this process.  The step
sweep is advice for the run config (``micro_batch_size``, ``model.loss_chunk_tokens``) and is
recorded, not applied.

    python -m tensor_train_ing_b200.tune attention --batch 8 --context 2048 --heads 16 --head-dim 128
    python -m tensor_train_ing_b200.tune gemm --shape 16384x10240x2048 --shape 16384x2048x8192
    python -m tensor_train_ing_b200.tune step --preset bench_1b --context 2048 --micro-batch 4 8 --loss-chunk 4096 8192
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

ATTENTION_GRIDS = (0, 148, 144, 140, 136, 132, 128, 120, 112, 96)  # 0: one CTA per SM
GEMM_TILES = (128, 256)


# ====================================================================================== timing
def _time_ms(fn, reps: int) -> float:
    """Mean milliseconds of ``fn`` over ``reps`` calls, L2 flushed before each."""
    flush = torch.empty(64 << 20, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        total += start.elapsed_time(end)
    return total / reps


def _lib():
    from .ops._ext import lib
    return lib()


def _ranked(rows: list[dict], key: str) -> list[dict]:
    return sorted(rows, key=lambda r: (not math.isfinite(r[key]), r[key]))


# ====================================================================================== attention
def _attention_inputs(batch, context, heads, head_dim, doc_len, seed=0):
    from .ops import fused
    from .ops.block import rope_context
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = batch * context
    positions = torch.arange(context, device="cuda")
    docs = (positions // doc_len if doc_len > 0 else torch.zeros_like(positions)).expand(batch, -1).contiguous()
    tables = fused.attention_tables(docs)
    width = heads * head_dim
    qkv = (torch.randn(n, 5 * width, device="cuda", generator=g) * 0.5).bfloat16()
    dout = torch.randn(n, width, device="cuda", generator=g).bfloat16()
    rope = rope_context(tables["pos32"], context, head_dim, 10000.0)
    return {"tables": tables, "qkv": qkv, "dout": dout, "rope": rope, "rs": torch.ones(n, device="cuda"),
            "par": torch.zeros(heads, 4, device="cuda"), "cols": [i * width for i in range(5)]}


def sweep_attention(batch=8, context=2048, heads=16, head_dim=128, doc_len=0, grids=ATTENTION_GRIDS,
                    reps=10) -> list[dict]:
    """Forward + backward time of the signed-product kernels for each grid limit (0: all SMs)."""
    C = _lib()
    x = _attention_inputs(batch, context, heads, head_dim, doc_len)
    t = x["tables"]

    def run():
        C.poly_fwd(0, head_dim, head_dim, x["qkv"], x["cols"], t["pos32"], t["doc32"], x["rs"], x["par"], batch,
                   context, heads)
        C.poly_bwd(0, head_dim, head_dim, x["qkv"], x["cols"], x["dout"], t["pos32"], t["doc32"], t["doc_end32"],
                   x["rs"], x["par"], batch, context, heads, x["rope"]["cos"], x["rope"]["sin"])
    rows = []
    try:
        for grid in grids:
            C.attn_grid_limit(int(grid))
            rows.append({"grid_limit": int(grid), "ms": _time_ms(run, reps)})
    finally:
        C.attn_grid_limit(0)
    from .ops._ext import check_status
    check_status()
    return _ranked(rows, "ms")


# ====================================================================================== gemm
def parse_shape(text: str) -> tuple[int, int, int]:
    parts = [int(v) for v in text.lower().split("x")]
    if len(parts) != 3 or min(parts) <= 0:
        raise ValueError(f"GEMM shape must be MxNxK with positive extents: {text!r}")
    return parts[0], parts[1], parts[2]


def sweep_gemm(shape, tiles=GEMM_TILES, reps=10) -> list[dict]:
    """bf16 [M, K] x [K, N] -> fp32 [M, N] time per tile width, with its TFLOP/s."""
    C = _lib()
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = torch.randn(N, K, device="cuda", generator=g).bfloat16().t()
    out = torch.empty(M, N, device="cuda")
    rows, first = [], None
    for tile in tiles:
        ms = _time_ms(lambda tile=tile: C.mm(a, b, out, None, 1.0, 0.0, None, None, int(tile)), reps)
        if first is None:
            first = out.clone()
        elif not torch.equal(first, out):  # every tile accumulates each element in the same K order
            raise RuntimeError(f"GEMM tile {tile} disagrees with tile {tiles[0]} at {shape}")
        rows.append({"shape": f"{M}x{N}x{K}", "tile_n": int(tile), "ms": ms,
                     "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12})
    return _ranked(rows, "ms")


# ====================================================================================== whole step
def sweep_step(preset="bench_1b", context=2048, rows_per_step=64, micro_batches=(4, 8, 16), loss_chunks=(4096, 8192),
               steps=2, optimizer="muon") -> list[dict]:
    """Tokens/s of full training steps (forward, backward, optimizer) per (micro-batch, CE chunk)."""
    from .config import Config, TrainConfig
    from .engine import TrainEngine
    from .models.shapes import preset as model_preset
    vocab = 50257
    out = []
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, vocab, (rows_per_step, context + 1), generator=g)
    idx = toks[:, :-1].pin_memory()
    targets = toks[:, 1:].contiguous().pin_memory()
    docs = torch.zeros_like(idx).pin_memory()
    for mb in micro_batches:
        for chunk in loss_chunks:
            model_cfg = model_preset(preset, loss_chunk_tokens=int(chunk))
            cfg = Config(model=model_cfg, train=TrainConfig(optimizer=optimizer, compile=False), raw={})
            try:
                engine = TrainEngine(cfg, device="cuda", micro_batch=int(mb), init="device")
                ms = _time_ms(lambda: engine.step(idx, docs, targets), steps)
                out.append({"micro_batch": int(mb), "loss_chunk_tokens": int(chunk), "ms_per_step": ms,
                            "tokens_per_second": rows_per_step * context / (ms * 1e-3)})
            except torch.OutOfMemoryError:
                out.append({"micro_batch": int(mb), "loss_chunk_tokens": int(chunk), "ms_per_step": math.inf,
                            "tokens_per_second": 0.0, "note": "out of memory"})
            finally:
                engine = None
                torch.cuda.empty_cache()
    return _ranked(out, "ms_per_step")


# ====================================================================================== results
def merge_best(path, kind: str, rows: list[dict], context: dict) -> dict:
    """Fold a sweep's best choice into the JSON file at ``path`` (created if absent)."""
    path = Path(path)
    table = json.loads(path.read_text()) if path.exists() else {}
    table.setdefault("gpu", torch.cuda.get_device_name() if torch.cuda.is_available() else None)
    best = rows[0]
    if kind == "attention":
        table["attention_grid_limit"] = best["grid_limit"]
        table["attention_context"] = context
    elif kind == "gemm":
        table.setdefault("gemm_tiles", {})[best["shape"]] = best["tile_n"]
    else:
        table.setdefault("step_advice", []).append({**context, "best": best})
    path.write_text(json.dumps(table, indent=2, sort_keys=True) + "\n")
    return table


def apply(source) -> dict:
    """Install a tuning table (a path or a dict): the attention grid limit and per-shape GEMM tiles."""
    table = json.loads(Path(source).read_text()) if isinstance(source, (str, Path)) else dict(source)
    from .ops import fused
    tiles = {}
    for shape, tile in (table.get("gemm_tiles") or {}).items():
        if tile not in GEMM_TILES:
            raise ValueError(f"GEMM tile must be one of {GEMM_TILES}: {shape} -> {tile}")
        tiles[parse_shape(shape)] = int(tile)
    fused.GEMM_TILES.clear()
    fused.GEMM_TILES.update(tiles)
    limit = table.get("attention_grid_limit")
    if limit is not None:
        if type(limit) is not int or limit < 0:
            raise ValueError("attention_grid_limit must be a nonnegative integer")
        if torch.cuda.is_available():
            _lib().attn_grid_limit(limit)
    return {"gemm_tiles": len(tiles), "attention_grid_limit": limit}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = p.add_subparsers(dest="kind", required=True)
    a = sub.add_parser("attention")
    a.add_argument("--batch", type=int, default=8)
    a.add_argument("--context", type=int, default=2048)
    a.add_argument("--heads", type=int, default=16)
    a.add_argument("--head-dim", type=int, default=128, choices=[64, 128])
    a.add_argument("--doc-len", type=int, default=0, help="0: one document per row")
    a.add_argument("--grids", type=int, nargs="+", default=list(ATTENTION_GRIDS))
    g = sub.add_parser("gemm")
    g.add_argument("--shape", action="append", required=True, help="MxNxK")
    s = sub.add_parser("step")
    s.add_argument("--preset", default="bench_1b")
    s.add_argument("--context", type=int, default=2048)
    s.add_argument("--rows", type=int, default=64, help="sequences per timed step")
    s.add_argument("--micro-batch", type=int, nargs="+", default=[4, 8, 16])
    s.add_argument("--loss-chunk", type=int, nargs="+", default=[4096, 8192])
    s.add_argument("--optimizer", default="muon", choices=["muon", "adamw"])
    for q in (a, g, s):
        q.add_argument("--reps", type=int, default=10)
        q.add_argument("--write", help="merge the best choice into this JSON file")
    args = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("tuning needs a CUDA device")
    report = {"gpu": torch.cuda.get_device_name(), "kind": args.kind}
    if args.kind == "attention":
        ctx = {"batch": args.batch, "context": args.context, "heads": args.heads, "head_dim": args.head_dim,
               "doc_len": args.doc_len}
        rows = sweep_attention(**ctx, grids=tuple(args.grids), reps=args.reps)
        report.update(context=ctx, rows=rows)
        if args.write:
            merge_best(args.write, "attention", rows, ctx)
    elif args.kind == "gemm":
        report["shapes"] = []
        for text in args.shape:
            rows = sweep_gemm(parse_shape(text), reps=args.reps)
            report["shapes"].append(rows)
            if args.write:
                merge_best(args.write, "gemm", rows, {})
    else:
        ctx = {"preset": args.preset, "context": args.context, "rows": args.rows, "optimizer": args.optimizer}
        rows = sweep_step(args.preset, args.context, args.rows, tuple(args.micro_batch), tuple(args.loss_chunk),
                          steps=args.reps, optimizer=args.optimizer)
        report.update(context=ctx, rows=rows)
        if args.write:
            merge_best(args.write, "step", rows, ctx)
    print(json.dumps(report, indent=1, default=str))
    return report


if __name__ == "__main__":
    main()
