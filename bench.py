"""Training-throughput benchmark: tokens/s of full training steps (fwd + bwd + Muon/AdamW update).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1b|7b|32b|100m|tiny] [--impl ours|reference]
                    [--shard-params auto|on|off] [--global-batch B] [--micro-batch M] [--no-e2e]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N ...

Default workload (the "~1B pilot" configuration): d_model 2048, 24 layers, 16 heads x 128, signed-product
polynomial attention, bilinear MLP 8192, pre-RMSNorm, vocab 50257 (padded 50304), T = 2048,
global batch 512 sequences (1,048,576 tokens) per optimizer step, chunked linear-CE with
8192-token chunks, Muon on hidden matrices + AdamW elsewhere, bf16 compute / fp32 master weights
and optimizer state.  Data: iid uniform token ids from a seed, next-token targets; random init.
The global batch is fixed, so runs at different N are strong scaling.  ``--config 7b`` / ``32b``
select the larger configurations (activation checkpointing; 32B needs parameter sharding over 8
GPUs, chosen automatically).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and a device synchronise on
both sides and timed with CUDA events on the launching stream; the reported time is the max over
ranks.  Every step's inputs (tens of MB of token ids) are copied from pinned host memory inside
the timed region; the per-step working set (weights, activations) is far larger than the 126 MB
L2, so no explicit flush is needed.  A separate end-to-end run through ``TrainEngine.step`` times
host wall clock and reads each step's loss back to the host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))

PRESETS = {
    # name: (layers, d_model, heads, head_dim, d_mlp, T, global_batch, micro_batch, act_ckpt, loss_chunk)
    "1b": (24, 2048, 16, 128, 8192, 2048, 512, 8, False, 8192),
    "7b": (32, 4096, 32, 128, 16384, 4096, 256, 4, True, 8192),
    "32b": (48, 6144, 48, 128, 24576, 4096, 256, 2, True, 8192),
    "100m": (12, 768, 12, 64, 3072, 2048, 256, 16, False, 8192),
    "tiny": (4, 256, 4, 64, 1024, 256, 8, 8, False, 0),
}
METRIC = "train tokens/s (8×B200, max over ranks) 1B/7B at 1/2/4/8 GPUs; MFU"


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", default="1b", choices=sorted(PRESETS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--micro-batch", type=int, default=None)
    p.add_argument("--optimizer", default="muon", choices=["muon", "adamw"])
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--recompute-blocks", default=None,
                   help="activation-checkpointed configs: recompute only the first N blocks, or 'auto' "
                        "(from the capacity plan and the GPU's memory; default: all)")
    p.add_argument("--global-batch", type=int, default=None,
                   help="override the preset's global batch (functional runs; the JSON line reports it)")
    p.add_argument("--shard-params", default="auto", choices=["auto", "on", "off"],
                   help="fp32 weights/grads/optimizer state only on owner ranks (auto: when replicated does not fit)")
    return p.parse_args()


def model_kwargs(name):
    L, d, H, hd, m, T, gb, mb, ckpt, chunk = PRESETS[name]
    vocab, padded = (4096, 4096) if name == "tiny" else (50257, 50304)
    return dict(layers=L, d_model=d, heads=H, d_key=hd, d_value=hd, d_mlp=m, vocab_size=vocab, padded_vocab=padded,
                attention="signed_product", mlp="bilinear", normalization="pre_rms",
                activation_checkpointing=ckpt, loss_chunk_tokens=chunk), T, gb, mb


def train_kwargs(opt):
    return dict(optimizer=opt, lr=6e-3 if opt == "muon" else 4.5e-4, aux_adamw_lr=4.5e-4, grad_clip=1.0,
                muon_adjust_lr="match_rms_adamw")


def setup_dist(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch N>1 with torchrun")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    return rank, world, torch.device("cuda", local)


def make_batches(steps, global_batch, T, vocab, rank, world, seed=0):
    """Uniform token ids; rank r takes rows [r*B/N, (r+1)*B/N) of every global batch."""
    g = torch.Generator().manual_seed(seed)
    rows = global_batch // world
    out = []
    for _ in range(steps):
        toks = torch.randint(0, vocab, (global_batch, T + 1), generator=g)[rank * rows:(rank + 1) * rows]
        idx = toks[:, :T].contiguous().pin_memory()
        tgt = toks[:, 1:].contiguous().pin_memory()
        docs = torch.zeros(rows, T, dtype=torch.long).pin_memory()
        out.append((idx, docs, tgt))
    return out


class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, devices):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in devices:
                continue
            try:
                mhz.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(mhz)}


def repo_libraries_loaded() -> list[str]:
    """Shared objects under this repository that the current process has mapped (/proc/self/maps)."""
    found = set()
    try:
        with open("/proc/self/maps") as fh:
            for line in fh:
                path = line.split()[-1] if len(line.split()) >= 6 else ""
                if path.startswith(ROOT) and ".so" in os.path.basename(path):
                    found.add(os.path.relpath(path, ROOT))
    except OSError:
        pass
    return sorted(found)


class _NoCounter:
    """The reference arm counts no kernels: this repository's library must stay out of its process."""
    count = None
    by_name = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def max_over_ranks(x, world, device):
    t = torch.tensor([x], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------ ours
def build_ours(args, device, world):
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.engine import TrainEngine
    mk, T, gb, mb = model_kwargs(args.config)
    cfg = Config.from_dict({"model": mk, "train": train_kwargs(args.optimizer)})
    torch.manual_seed(101)
    shard = {"auto": None, "on": True, "off": False}[args.shard_params]
    if shard is None:
        from tensor_train_ing_b200.models.shapes import needs_parameter_sharding
        shard = needs_parameter_sharding(cfg.model, world, device)
    # a sharded model is drawn on the device (the serial CPU initialisation of 33B weights takes minutes)
    eng = TrainEngine(cfg, device=device, micro_batch=args.micro_batch or mb, shard_params=shard,
                      init="device" if shard else "serial",
                      recompute_blocks=(args.recompute_blocks if args.recompute_blocks in (None, "auto")
                                        else int(args.recompute_blocks)))
    if not eng.fused:
        raise SystemExit("the fused sm_100a path does not cover this configuration")
    n_params = sum(p.numel() for p in eng.model.parameters())

    def step(batch):
        loss, count = eng.step(*batch)
        return loss, count

    return step, cfg, T, gb, n_params, eng


# ------------------------------------------------------------------------------------------ reference
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def install_reference() -> str:
    """Install the unmodified reference package into baseline/_ref if it is not there yet.

    The reference pins a torch release the offline wheelhouse does not carry, so dependency
    resolution fails; with ``--no-deps`` the package installs and runs on the image's torch.  The
    source directory comes from ``TTB_REFERENCE_SRC`` or BASELINE.json's ``reference_path``; it is
    copied to a temporary directory first because the build writes into its source tree.
    """
    if os.path.isdir(os.path.join(REF_DIR, "tnlm")):
        return REF_DIR
    src = os.environ.get("TTB_REFERENCE_SRC")
    if not src:
        try:
            with open(os.path.join(ROOT, "BASELINE.json")) as fh:
                src = json.load(fh).get("reference_path")
        except (OSError, ValueError):
            src = None
    if not src or not os.path.isdir(src):
        raise RuntimeError(f"reference not installed in {os.path.relpath(REF_DIR, ROOT)} and its source "
                           f"({src or 'no reference_path'}) is not on this machine")
    import shutil
    import tempfile
    wheels = os.environ.get("TTB_WHEELHOUSE", "/opt/wheelhouse")
    with tempfile.TemporaryDirectory() as tmp:
        copy = os.path.join(tmp, "src")
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", wheels, "--target", REF_DIR, copy]
        proc = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    if proc.returncode != 0 or not os.path.isdir(os.path.join(REF_DIR, "tnlm")):
        tail = (proc.stderr or proc.stdout).strip().splitlines()[-1:] or ["no output"]
        raise RuntimeError(f"pip install --no-deps of the reference failed: {tail[0]}")
    return REF_DIR


def build_reference(args, device, world):
    error = None
    rank = dist.get_rank() if world > 1 else 0
    if rank == 0:
        try:
            install_reference()
        except Exception as e:  # reported by every rank below, after the others learn of it
            error = f"{type(e).__name__}: {e}"
    if world > 1:
        box = [error]
        dist.broadcast_object_list(box, src=0)
        error = box[0]
    if error:
        raise RuntimeError(error)
    ref = REF_DIR
    if args.config == "32b":
        raise RuntimeError("the reference's stock bench path builds the full fp32 32B model on every rank's CPU "
                           "(133 GB per rank, over 1 TB for 8 ranks)")
    sys.path.insert(0, ref)
    from tnlm.config import ModelConfig, TrainConfig
    from tnlm.model import TensorLM
    from tnlm.optim import make_optimizer
    from tnlm.parallel import global_count, shard_model
    mk, T, gb, mb = model_kwargs(args.config)
    mcfg = ModelConfig(**mk)
    tcfg = TrainConfig(**train_kwargs(args.optimizer))
    torch.manual_seed(101)
    model = TensorLM(mcfg).to(device)
    if world > 1:
        from torch.distributed.device_mesh import init_device_mesh
        mesh = init_device_mesh("cuda", (world,))
        model = shard_model(model, mesh)
    opt = make_optimizer(model, tcfg)
    # the reference's serial trainer compiles the model when train.compile is set (its default;
    # tnlm/train.py:353); its distributed trainer does not compile
    forward = model
    compile_note = "eager (the reference's distributed trainer does not compile)"
    if world == 1 and tcfg.compile:
        forward = torch.compile(model)
        compile_note = "torch.compile(model), as the reference's serial trainer"
    n_params = sum(p.numel() for p in model.parameters())
    if world > 1:
        n_params = sum(p.full_tensor().numel() if hasattr(p, "full_tensor") else p.numel() for p in model.parameters())
    micro = args.micro_batch or mb

    def step(batch):
        idx, docs, tgt = batch
        opt.zero_grad(set_to_none=True)
        count = global_count((tgt != -100).sum().to(device))
        total = torch.zeros((), device=device)
        for s in range(0, idx.shape[0], micro):
            i, d, t = (x[s:s + micro].to(device, non_blocking=True) for x in (idx, docs, tgt))
            with torch.autocast("cuda", dtype=torch.bfloat16):
                _, loss, _ = forward(i, doc_ids=d, targets=t, reduction="sum")
            (loss / count).backward()
            total += loss.detach().float()
        torch.nn.utils.clip_grad_norm_(model.parameters(), tcfg.grad_clip)
        opt.step()
        if world > 1:
            dist.all_reduce(total)
        return total, count

    step.note = compile_note
    return step, mcfg, T, gb, n_params, None


def main():
    args = parse()
    rank, world, device = setup_dist(args.gpus)
    if args.warmup < 3 and rank == 0:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    try:
        builder = build_ours if args.impl == "ours" else build_reference
        step, cfg, T, gb, n_params, eng = builder(args, device, world)
        if args.global_batch is not None:
            if args.global_batch % world:
                raise SystemExit("--global-batch must be a multiple of the GPU count")
            gb = args.global_batch
    except Exception as e:  # the reference may not build/run on this stack; say so in one line
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(e).__name__}: {e}"[:300]}))
            if world > 1:
                dist.destroy_process_group()
            return
        raise
    vocab = 4096 if args.config == "tiny" else 50257
    batches = make_batches(args.warmup + args.steps, gb, T, vocab, rank, world)
    tokens_per_step = gb * T

    try:
        for i in range(args.warmup):
            step(batches[i])
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        # ------------------------------------------------------------ device-timed region
        if args.impl == "ours":
            from tensor_train_ing_b200.ops._ext import launch_counter
            eng.phase_events = []
        else:
            launch_counter = _NoCounter
        sampler = ClockSampler()
        if rank == 0:
            sampler.start()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with launch_counter() as counter:
            start.record()
            losses = []
            for i in range(args.steps):
                loss, count = step(batches[args.warmup + i])
                losses.append(loss)
            stop.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
        phases = eng.phase_times_ms() if eng is not None else {}
        if eng is not None:
            eng.phase_events = None
        ms = max_over_ranks(ms, world, device)
        # per-phase device time, max over ranks (the phases run back to back on the compute stream)
        phases = {k: round(max_over_ranks(v, world, device), 2) for k, v in sorted(phases.items())}
        clocks = sampler.stop(set(range(world))) if rank == 0 else None
        loss_vals = [float(l) / tokens_per_step for l in losses]
        ms_per_step = ms / args.steps
        value = tokens_per_step / (ms_per_step / 1000.0)

        # ------------------------------------------------------------ end-to-end (public API, host clock)
        e2e = None
        if not args.no_e2e:
            e2e_steps = max(1, min(args.steps, 2))
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            for i in range(e2e_steps):
                loss, count = step(batches[args.warmup + (i % args.steps)])
                float(loss.item())  # device -> host read of the step's result
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            wall = max_over_ranks(time.perf_counter() - t0, world, device)
            idx0 = batches[0][0]
            h2d = 3 * idx0.numel() * idx0.element_size()
            e2e = {"value": tokens_per_step * e2e_steps / wall, "unit": "tokens/s",
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                   "api": "TrainEngine.step" if args.impl == "ours" else "tnlm TensorLM/make_optimizer loop"}
    except torch.OutOfMemoryError as e:
        # the reference's stock path may not fit a configuration on one GPU (7B at micro-batch 4): say so
        # in one line; a multi-rank run ends through torchrun, whose other ranks stop with this one
        if args.impl != "reference" or world > 1:
            raise
        print(json.dumps({"impl": "reference", "unavailable": f"out of memory: {str(e).splitlines()[0]}"[:300],
                          "config": {"model": f"tnlm-{args.config}", "micro_batch": args.micro_batch}}))
        return

    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak_tflops, sustained_tflops = 1590.0, 1400.0
    if os.path.exists(peaks_path):
        with open(peaks_path) as fh:
            peaks = json.load(fh)
        peak_tflops = float(peaks.get("bf16_tflops", peak_tflops))
        sustained_tflops = float(peaks.get("bf16_tflops_sustained", sustained_tflops))
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic uniform token ids (seed 0), next-token targets; random init weights",
            "config": {"model": f"tnlm-{args.config}", "global_batch": gb, "seq_len": T,
                       "parallelism": f"dp{world}" + ("-param-sharded" if eng is not None and eng.shard_params
                                                       else ""), "tokens_per_step": tokens_per_step,
                       "optimizer": f"{args.optimizer} (hidden) + adamw", "micro_batch": args.micro_batch
                       or PRESETS[args.config][7], "params": n_params,
                       "l2": "per-step working set >> 126 MB L2; no flush needed",
                       "recompute_blocks": (getattr(eng.model, "recompute_blocks", None) if eng is not None
                                            else None)},
            "mfu": round(6 * n_params * value / (world * peak_tflops * 1e12), 4),
            "mfu_peak_tflops": peak_tflops,
            "mfu_of_sustained": round(6 * n_params * value / (world * sustained_tflops * 1e12), 4),
            "mfu_sustained_tflops": sustained_tflops,
            "loss_first_last": [round(loss_vals[0], 4), round(loss_vals[-1], 4)],
            "clocks": clocks, "e2e": e2e,
            "peak_mem_gb": round(torch.cuda.max_memory_allocated(device) / 1e9, 1),
        }
        if args.impl == "reference":
            out["impl"] = "reference"
            out["config"]["reference_path"] = getattr(step, "note", None)
        else:
            out["gpu_launches"] = counter.count
            out["gpu_launches_by_binding"] = counter.by_name
            out["phase_ms_per_step"] = phases
        out["native_so_loaded"] = repo_libraries_loaded()
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
