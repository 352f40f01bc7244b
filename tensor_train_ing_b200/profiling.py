"""Per-update kernel profiling: CUDA device time per kernel name, NVTX-style named regions and
Chrome-trace export (reference tnlm/profiling.py:13-136).

``KernelProfile(warmup_steps, ...)`` is driven by a trainer through ``start_step`` /
``finish_step`` / ``region(name)``; after warm-up it captures ``trace_steps`` updates with
``torch.profiler`` (CUDA activity) and sums raw device kernel time by kernel name, excluding
user annotations, so the report ranks kernels by their share of the step.  Times taken under a
profiler are for shares and rankings only, never for throughput numbers.
"""
from __future__ import annotations

import json
import os
import tempfile
from contextlib import contextmanager, nullcontext
from pathlib import Path

import torch


def _kernel_events(prof):
    rows = {}
    for evt in prof.events():
        dev_type = getattr(evt, "device_type", None)
        if dev_type is None or "CUDA" not in str(dev_type):
            continue
        if getattr(evt, "is_user_annotation", False):
            continue
        name = evt.name
        dur = getattr(evt, "device_time", None)
        if dur is None:
            dur = getattr(evt, "cuda_time", 0.0)
        r = rows.setdefault(name, {"name": name, "count": 0, "total_us": 0.0})
        r["count"] += 1
        r["total_us"] += float(dur)
    return sorted(rows.values(), key=lambda r: -r["total_us"])


class KernelProfile:
    def __init__(self, warmup_steps: int = 2, trace_dir: str | os.PathLike | None = None, trace_steps: int = 1,
                 cuda: bool = True, kernels: bool = True, nvtx: bool = True):
        self.warmup_steps = int(warmup_steps)
        self.trace_steps = max(1, int(trace_steps))
        self.trace_dir = Path(trace_dir) if trace_dir else None
        self.cuda = cuda
        self.kernels = kernels
        self.nvtx = nvtx and cuda and torch.cuda.is_available()
        self._prof = None
        self._step = None
        self._captured = 0
        self.rows: list[dict] = []
        self.steps: list[int] = []

    def _active(self):
        return self._step is not None and self._step >= self.warmup_steps and self._captured < self.trace_steps

    def start_step(self, step: int):
        self._step = step
        if self._active() and self._prof is None:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if self.cuda:
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self._prof = torch.profiler.profile(activities=acts, record_shapes=False)
            self._prof.__enter__()

    def finish_step(self):
        if self._prof is None or not self._active():
            return
        if self.cuda:
            torch.cuda.synchronize()
        self.steps.append(self._step)
        self._captured += 1
        if self._captured >= self.trace_steps:
            self._stop()

    def _stop(self):
        prof, self._prof = self._prof, None
        prof.__exit__(None, None, None)
        if self.kernels:
            self.rows = _kernel_events(prof)
        if self.trace_dir is not None:
            self.trace_dir.mkdir(parents=True, exist_ok=True)
            fd, tmp = tempfile.mkstemp(dir=self.trace_dir, suffix=".json.tmp")
            os.close(fd)
            prof.export_chrome_trace(tmp)
            os.replace(tmp, self.trace_dir / f"trace-steps-{self.steps[0]}-{self.steps[-1]}.json")

    @contextmanager
    def region(self, name: str):
        ctx = torch.profiler.record_function(name) if self._prof is not None else nullcontext()
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        try:
            with ctx:
                yield
        finally:
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    def report(self, top: int = 40) -> dict:
        total = sum(r["total_us"] for r in self.rows) or 1.0
        return {"captured_steps": self.steps, "kernel_total_ms": total / 1000.0,
                "kernels": [{**r, "share": r["total_us"] / total} for r in self.rows[:top]]}

    def close(self):
        if self._prof is not None:
            self._stop()


def profile_callable(fn, warmup: int = 1, repeat: int = 1, top: int = 30) -> dict:
    """Profile ``fn()`` after ``warmup`` calls; returns the kernel-time table."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    prof = KernelProfile(warmup_steps=0, trace_steps=repeat)
    for i in range(repeat):
        prof.start_step(i)
        fn()
        prof.finish_step()
    prof.close()
    return prof.report(top)


def main(argv=None):  # pragma: no cover - GPU tool
    import argparse
    p = argparse.ArgumentParser(description="kernel-time breakdown of one training step of a bench preset")
    p.add_argument("--config", default="1b")
    p.add_argument("--rows", type=int, default=16, help="sequences in the profiled step")
    p.add_argument("--micro-batch", type=int, default=8)
    p.add_argument("--out", default=None)
    a = p.parse_args(argv)
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from .config import Config
    from .engine import TrainEngine
    mk, T, _, _ = bench.model_kwargs(a.config)
    cfg = Config.from_dict({"model": mk, "train": bench.train_kwargs("muon")})
    eng = TrainEngine(cfg, device="cuda", micro_batch=a.micro_batch)
    (batch,) = bench.make_batches(1, a.rows, T, mk["vocab_size"], 0, 1)
    rep = profile_callable(lambda: eng.step(*batch), warmup=2, repeat=1)
    text = json.dumps(rep, indent=1)
    if a.out:
        Path(a.out).write_text(text)
    print(text)


if __name__ == "__main__":  # pragma: no cover
    main()
