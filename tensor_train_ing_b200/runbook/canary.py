"""Day-one canary for a B200 box: kernel numerics spot checks, then full training steps of a
benchmark shape gated on throughput (the reference's scripts/h100_canary.py role).

    python -m tensor_train_ing_b200.runbook.canary --out runs/canary [--preset bench_1b] [--steps 20]
        [--min-tok-s 60000] [--warmup-steps 3]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m tensor_train_ing_b200.runbook.canary --out ...

1. Numerics: the tcgen05 GEMM, polynomial attention (forward and backward), RMSNorm and fused
   cross-entropy against PyTorch fp32 / fp64 evaluations on small cases; a failure stops the
   canary before any throughput is measured.
2. Throughput: ``TrainEngine`` steps (forward, backward, Muon/AdamW update) on synthetic uniform
   tokens, each step timed with CUDA events on the launching stream and the maximum over ranks
   taken; the first ``--warmup-steps`` are excluded and the rest feed ``ThroughputCanary``, which
   fails when the rate is below ``--min-tok-s``.  Losses must stay finite.
3. Report (rank 0): pass/fail, the per-step rates, an MFU estimate (6 x parameters x tokens/s over
   the measured bf16 GEMM peak in ``MEASURED_PEAKS.json`` or ``--peak-tflops``), peak memory per
   rank and the clocks seen, as ``result.json`` in ``--out``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[2]


# ====================================================================================== numerics
def _rel(got, want) -> float:
    got, want = got.double(), want.double()
    return float((got - want).norm() / want.norm().clamp_min(1e-30))


def numerics_checks() -> list[dict]:
    """Each hot kernel family against a PyTorch fp32 / fp64 evaluation at a small shape: relative
    Frobenius error below 3e-2 (bf16 operands), 1e-3 for the fp32 cross-entropy."""
    from ..ops import fused
    from ..ops._ext import check_status, lib
    C = lib()
    g = torch.Generator(device="cuda").manual_seed(0)
    out = []

    def record(name, err, bound):
        out.append({"check": name, "relative_error": err, "bound": bound, "ok": err < bound})
    a = torch.randn(384, 512, device="cuda", generator=g).bfloat16()
    b = torch.randn(640, 512, device="cuda", generator=g).bfloat16()
    record("gemm", _rel(fused._mm(a, b.t(), torch.empty(384, 640, device="cuda")), a.float() @ b.float().t()), 3e-2)
    x = torch.randn(256, 1024, device="cuda", generator=g)
    w = 1 + 0.1 * torch.randn(1024, device="cuda", generator=g)
    y, _ = C.rmsnorm_fwd(x, w, 1, 1e-6)
    record("rmsnorm", _rel(y, x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w), 3e-2)
    xs = (torch.randn(256, 512, device="cuda", generator=g) * 0.5).bfloat16()
    ws = (torch.randn(1024, 512, device="cuda", generator=g) * 0.05).bfloat16()
    t = torch.randint(0, 1000, (256,), device="cuda", generator=g)
    loss, _ = C.ce_fwd(xs, ws, 1000, 1.0, t, torch.empty(256, 1024, device="cuda"))
    want = torch.nn.functional.cross_entropy((xs.float() @ ws.float().t())[:, :1000], t, reduction="none")
    record("cross_entropy", _rel(loss, want), 1e-3)
    record("polynomial_attention_fwd_bwd", _attention_error(fused), 3e-2)
    check_status()
    return out


def _attention_error(fused) -> float:
    """Largest relative error of the signed-product attention output and input gradient against
    the dense fp64 oracle (two rows of two documents each, row scale power 1/2)."""
    from ..models.attention import polynomial_attention, row_scale_mask, row_scale_vector, visible_mask
    B, T, H, dk = 2, 256, 2, 128
    g = torch.Generator(device="cuda").manual_seed(1)
    cols = [i * H * dk for i in range(5)]
    qkv = (torch.randn(B * T, 5 * H * dk, device="cuda", generator=g) * 0.7).bfloat16().requires_grad_()
    docs = (torch.arange(T, device="cuda") >= 100).long().expand(B, -1).contiguous()
    tables = fused.attention_tables(docs)
    y = fused.poly_attention(qkv, None, "signed_product", dk, dk, H, cols, tables,
                             row_scale_vector(docs, 0.5).contiguous().view(-1))
    gy = torch.randn(y.shape, device="cuda", generator=g)
    y.backward(gy.to(y.dtype))
    ref = qkv.detach().double().requires_grad_()
    q1, k1, q2, k2, v = (ref[:, c:c + H * dk].view(B, T, H, dk).transpose(1, 2) for c in cols)
    want = polynomial_attention("signed_product", q1, k1, q2, k2, v,
                                row_scale_mask(visible_mask(docs), 0.5, dtype=torch.float64))
    want = want.transpose(1, 2).reshape(B * T, H * dk)
    want.backward(gy.double())
    return max(_rel(y.float(), want), _rel(qkv.grad.float(), ref.grad))


# ====================================================================================== throughput
def _peak_tflops(override):
    if override:
        return float(override)
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"])
    except (OSError, KeyError, ValueError):
        return None


def _clocks(device_index: int) -> dict:
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
        return {"sm_mhz": pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                "sm_max_mhz": pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM),
                "throttle_reasons": int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))}
    except Exception as exc:  # clocks are informational
        return {"unavailable": type(exc).__name__}


def run_canary(out_dir, *, preset="bench_1b", context=2048, rows_per_rank=16, micro_batch=8, steps=20,
               warmup_steps=3, min_tokens_per_second=None, optimizer="muon", peak_tflops=None) -> dict | None:
    from ..config import Config, TrainConfig
    from ..engine import TrainEngine
    from ..models.shapes import count_params, preset as model_preset
    from ..throughput_canary import ThroughputCanary
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    out_dir = Path(out_dir)
    checks = numerics_checks()
    passed = torch.tensor([int(all(c["ok"] for c in checks))], device="cuda")
    if world > 1:  # every rank stops, or none does
        dist.all_reduce(passed, op=dist.ReduceOp.MIN)
    if not int(passed):
        report = {"status": "failed", "stage": "numerics", "numerics": checks}
        if rank == 0:
            out_dir.mkdir(parents=True, exist_ok=True)
            (out_dir / "result.json").write_text(json.dumps(report, indent=2) + "\n")
        return report if rank == 0 else None
    model_cfg = model_preset(preset)
    cfg = Config(model=model_cfg, train=TrainConfig(optimizer=optimizer, compile=False, lr=6e-3 if optimizer == "muon"
                                                    else 4.5e-4, aux_adamw_lr=4.5e-4), raw={})
    engine = TrainEngine(cfg, device=torch.device("cuda", torch.cuda.current_device()), micro_batch=micro_batch,
                         init="device")
    gen = torch.Generator().manual_seed(1234 + rank)
    tokens = rows_per_rank * context
    gate = (ThroughputCanary(steps - warmup_steps, float(min_tokens_per_second), warmup_steps)
            if min_tokens_per_second else None)
    rows = []
    for step in range(1, steps + 1):
        toks = torch.randint(0, model_cfg.vocab_size, (rows_per_rank, context + 1), generator=gen).pin_memory()
        docs = torch.zeros(rows_per_rank, context, dtype=torch.long)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record()
        loss, count = engine.step(toks[:, :-1], docs, toks[:, 1:])
        end.record()
        torch.cuda.synchronize()
        seconds = torch.tensor([start.elapsed_time(end) / 1e3], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(seconds, op=dist.ReduceOp.MAX)
        row = {"step": step, "loss": float(loss) / max(int(count), 1), "seconds": float(seconds),
               "prediction_tokens": tokens * world}
        if not math.isfinite(row["loss"]):
            raise FloatingPointError(f"non-finite loss at canary step {step}")
        rows.append(row)
        if gate is not None:
            gate.observe(row)
    memory = {"rank": rank, "peak_allocated_bytes": torch.cuda.max_memory_allocated(),
              "total_bytes": torch.cuda.get_device_properties(torch.cuda.current_device()).total_memory,
              "clocks": _clocks(torch.cuda.current_device())}
    memories = [None] * world
    if world > 1:
        dist.all_gather_object(memories, memory)
    else:
        memories = [memory]
    if rank != 0:
        return None
    measured = rows[warmup_steps:]
    rate = sum(r["prediction_tokens"] for r in measured) / sum(r["seconds"] for r in measured)
    params = count_params(model_cfg)["total"]
    peak = _peak_tflops(peak_tflops)
    report = {"status": "passed", "world_size": world, "preset": preset, "context": context, "optimizer": optimizer,
              "numerics": checks, "steps": rows, "warmup_steps_excluded": warmup_steps,
              "tokens_per_second": rate, "tokens_per_second_per_gpu": rate / world, "parameters_total": params,
              "mfu_estimate": 6 * params * rate / (world * peak * 1e12) if peak else None,
              "mfu_definition": "6 x total parameters x tokens/s / (GPUs x measured sustained bf16 GEMM peak); "
                                "attention FLOPs excluded",
              "memory_per_rank": memories,
              "throughput_gate": gate.require_complete() if gate is not None else None}
    out_dir.mkdir(parents=True, exist_ok=True)
    (out_dir / "result.json").write_text(json.dumps(report, indent=2, default=str) + "\n")
    return report


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--out", required=True)
    p.add_argument("--preset", default="bench_1b")
    p.add_argument("--context", type=int, default=2048)
    p.add_argument("--rows-per-rank", type=int, default=16)
    p.add_argument("--micro-batch", type=int, default=8)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup-steps", type=int, default=3)
    p.add_argument("--min-tok-s", type=float)
    p.add_argument("--optimizer", default="muon", choices=["muon", "adamw"])
    p.add_argument("--peak-tflops", type=float)
    a = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("the canary needs a CUDA device")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        local = int(os.environ["LOCAL_RANK"])
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    try:
        report = run_canary(a.out, preset=a.preset, context=a.context, rows_per_rank=a.rows_per_rank,
                            micro_batch=a.micro_batch, steps=a.steps, warmup_steps=a.warmup_steps,
                            min_tokens_per_second=a.min_tok_s, optimizer=a.optimizer, peak_tflops=a.peak_tflops)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
    if report is not None:
        print(json.dumps({k: report.get(k) for k in ("status", "tokens_per_second", "mfu_estimate")}))
        return 0 if report["status"] == "passed" else 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
