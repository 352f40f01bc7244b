"""Command line: ``tnlm COMMAND`` or ``python -m tensor_train_ing_b200.cli COMMAND``.

The subcommands and flags are the reference's (tnlm/cli.py:331-683) so existing configs, scripts
and run books keep working: validate_config, plan_search, sweep-config, sweep, reconcile,
prepare_data, prepare_mechanisms, evaluate_mechanisms, train, cooldown, branch, profile, analyze,
evaluate, record_spend, compare_evaluations, compare_seed_pairs, summarize, check_math.  Training
defaults to a configuration dry run (``project.dry_run``).  ``--distributed`` runs under torchrun,
one process per GPU over NCCL (gloo on CPU).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import shutil
from datetime import timedelta
from pathlib import Path

import torch

from .checkpoint_plan import checkpoint_storage_plan
from .config import Config
from .models.model import TensorLM
from .runtime import full_config
from .train import plan_search, profile_run, train_run


def _checkpoint_disk_check(storage_plan, run_dir=None):
    """Advisory projection of a fresh run's checkpoints against the destination filesystem now."""
    from .checkpoint_storage import RESERVE_BYTES
    dest = Path(run_dir).absolute() if run_dir is not None else Path.cwd()
    info = {"destination": str(dest), "destination_source": "run_dir" if run_dir is not None else "current_working_directory",
            "required_additional_bytes": storage_plan["required_additional_bytes"], "reserve_bytes": RESERVE_BYTES,
            "free_bytes": None, "filesystem_probe_path": None,
            "scope": "advisory fresh serial run projection; no reservation"}
    try:
        probe = dest
        while not probe.exists():
            if probe.parent == probe:
                raise FileNotFoundError(str(probe))
            probe = probe.parent
        info["filesystem_probe_path"] = str(probe)
        info["free_bytes"] = shutil.disk_usage(probe).free
    except OSError as e:
        info.update(status="unavailable", error=str(e))
        return info, [f"Checkpoint disk availability could not be checked: {e}"]
    if info["free_bytes"] < info["required_additional_bytes"] + RESERVE_BYTES:
        info["status"] = "insufficient"
        return info, [f"Checkpoint storage projection needs {info['required_additional_bytes']} bytes plus "
                      f"{RESERVE_BYTES} reserve, but only {info['free_bytes']} bytes are free on {probe}."]
    info["status"] = "ok"
    return info, []


def validate_config(cfg, device=None, run_dir=None) -> dict:
    """Parameter counts, operator audit, capacity plan and checkpoint storage projection, without
    allocating weights (the model is built on the meta device)."""
    from .models.shapes import memory_plan

    class ShapeOnly(TensorLM):
        def reset_parameters(self):
            pass
    with torch.device("meta"):
        model = ShapeOnly(cfg.model)
    counts = model.param_counts()
    audit = model.operator_audit()
    data = cfg.raw.get("data", {})
    context, batch = data.get("context", 512), data.get("micro_batch_size", 1)
    dev = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    fused, why = model.fused_path_supported()
    backend = cfg.model.attention_backend
    if backend == "auto":
        backend = "cuda" if dev.type == "cuda" and fused else "reference"
    if cfg.model.attention == "softmax":
        backend = "flex" if dev.type == "cuda" else "softmax"
    gpu_gb = (torch.cuda.get_device_properties(dev).total_memory / 1e9
              if dev.type == "cuda" and torch.cuda.is_available() else 180.0)
    capacity = memory_plan(cfg.model, gpus=1, micro_tokens_per_gpu=batch * context, gpu_gb=gpu_gb,
                           optimizer=cfg.train.optimizer)
    storage = checkpoint_storage_plan(cfg)
    disk, warnings = _checkpoint_disk_check(storage, run_dir)
    loss_rows = batch * context if cfg.model.loss_chunk_tokens <= 0 else min(batch * context, cfg.model.loss_chunk_tokens)
    return {"parameters": counts, "operator_audit": audit, "memory_plan": capacity,
            "checkpoint_storage_plan": storage, "checkpoint_disk_check": disk, "warnings": warnings,
            "memory_plan_assumptions": {"gpu_capacity_GB": gpu_gb,
                                        "capacity_source": "selected CUDA device" if dev.type == "cuda" and torch.cuda.is_available()
                                        else "hypothetical 180 GB B200"},
            "global_polynomial_degree_upper_bound": 10 ** cfg.model.layers if audit["class"] == "P" else None,
            "estimated_one_fp32_training_logit_chunk_bytes": loss_rows * cfg.model.vocab_size * 4,
            "scaling": {"default_training_world_size": 1,
                        "distributed_training": {"entrypoint": "train/cooldown --distributed under torchrun",
                                                 "layout": "owner-computes sharded data parallelism",
                                                 "supported_optimizers": ["adamw", "muon"],
                                                 "recovery_world_size": "must match checkpoint"},
                        "fused_sm100a_path": fused, "fused_path_limit": why or None,
                        "attention_backend": cfg.model.attention_backend, "resolved_attention_backend": backend,
                        "device": str(dev), "cuda_available": torch.cuda.is_available(),
                        "activation_checkpointing": cfg.model.activation_checkpointing,
                        "loss_chunk_tokens": cfg.model.loss_chunk_tokens},
            "weight_decay_policy": "hidden linear-map weights only; embeddings, output vocabulary, gains, biases "
                                   "and head scalars excluded",
            "config": full_config(cfg)}


def _distributed_run(cfg, args):
    """Initialise a bounded torchrun process group (NCCL on CUDA, gloo on CPU); rank 0 returns the result."""
    import torch.distributed as dist

    from .runtime import deterministic_execution, deterministic_requested
    timeout = args.collective_timeout_seconds
    if not math.isfinite(timeout) or timeout <= 0:
        raise ValueError("collective timeout must be finite and positive")
    context_fork = getattr(args, "context_fork", False)
    if context_fork and args.resume is None:
        raise ValueError("context_fork requires an explicit parent checkpoint")
    if cfg.raw.get("project", {}).get("dry_run", True):
        result = plan_search(cfg)
        result.update(distributed=True, collective_timeout_seconds=timeout, context_fork=context_fork,
                      parent=str(args.resume) if args.resume is not None else None,
                      launch="torchrun --standalone --nproc-per-node N -m tensor_train_ing_b200.cli train --distributed ...")
        return result if int(os.environ.get("RANK", "0")) == 0 else None
    owned = not dist.is_initialized()
    dev = torch.device(args.device)
    if owned:
        if any(k not in os.environ for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")):
            raise ValueError("--distributed requires a torchrun launch with rank/rendezvous environment")
        if dev.type == "cuda":
            if dev.index is not None:
                raise ValueError("use --device cuda so torchrun LOCAL_RANK selects each GPU")
            dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
            torch.cuda.set_device(dev)
        elif dev.type != "cpu":
            raise ValueError("distributed training supports CPU/gloo or CUDA/NCCL")
        dist.init_process_group("nccl" if dev.type == "cuda" else "gloo", timeout=timedelta(seconds=timeout))
    try:
        from .distributed_train import distributed_train_run
        with deterministic_execution(deterministic_requested(cfg), device=str(dev)):
            result = distributed_train_run(cfg, args.run_dir, max_steps=args.max_steps, max_seconds=args.max_seconds,
                                           device=str(dev), resume=args.resume, context_fork=context_fork,
                                           cooldown_steps=getattr(args, "cooldown_steps", None),
                                           cooldown_end_tokens=getattr(args, "cooldown_end_tokens", None),
                                           run_budget_usd=args.run_budget_usd,
                                           export_max_state_bytes=args.export_max_state_bytes,
                                           checkpoint_format=args.checkpoint_format)
        return result if dist.get_rank() == 0 else None
    finally:
        if owned:
            dist.destroy_process_group()


def _pairs_file(path, sides):
    import yaml
    pf = Path(path).resolve()
    pairs = yaml.safe_load(pf.read_text())
    if isinstance(pairs, list):
        for pair in pairs:
            if isinstance(pair, dict):
                for side in sides:
                    if isinstance(pair.get(side), str):
                        pair[side] = str((pf.parent / pair[side]).resolve())
    return pairs


def _parser():
    parser = argparse.ArgumentParser(prog="tnlm", description=__doc__.split("\n")[0])
    sub = parser.add_subparsers(dest="command", required=True)
    for name in ("validate_config", "plan_search"):
        p = sub.add_parser(name)
        p.add_argument("--config", required=True)
        if name == "plan_search":
            p.add_argument("--candidates", help="YAML/JSON list of named configuration overrides; planning only")
        else:
            p.add_argument("--device", help="resolve the attention backend for this device without allocating weights")
            p.add_argument("--run-dir", help="future checkpoint destination for the advisory free-disk check")
    p = sub.add_parser("sweep-config", help="export one recorded sweep candidate as YAML without training")
    p.add_argument("--sweep", required=True)
    p.add_argument("--candidate", required=True)
    p.add_argument("--out")
    p = sub.add_parser("sweep")
    p.add_argument("--config", required=True)
    p.add_argument("--candidates", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--max-seconds", type=float, required=True, help="runtime bound per training segment")
    p.add_argument("--evaluation-max-seconds", type=float, required=True)
    p.add_argument("--max-prediction-tokens", type=int, default=1_000_000)
    p.add_argument("--bootstrap-samples", type=int, default=1000)
    p.add_argument("--device", default="cuda")
    p.add_argument("--no-cooldown", action="store_true")
    p.add_argument("--reference-candidate")
    p.add_argument("--prune-completed-intermediates", action="store_true")
    p.add_argument("--canary-steps", type=int, default=0)
    p.add_argument("--min-tok-s", "--expect-tok-s", dest="min_tok_s", type=float)
    p.add_argument("--canary-warmup-steps", type=int, default=12)
    p.add_argument("--snapshot-sources", nargs="?", const="", metavar="DIR")
    p = sub.add_parser("reconcile", help="inspect or explicitly reconcile one terminal runtime ledger entry")
    p.add_argument("--ledger", required=True)
    p.add_argument("--run-id", required=True)
    p.add_argument("--metrics", action="append", default=[])
    p.add_argument("--apply", action="store_true")
    p.add_argument("--expected-row-sha256")
    p.add_argument("--operator")
    p.add_argument("--reason")
    p.add_argument("--all-workers-stopped", action="store_true")
    p.add_argument("--observed-elapsed-seconds", type=float)
    totals = p.add_mutually_exclusive_group()
    totals.add_argument("--total-elapsed-seconds", type=float)
    totals.add_argument("--total-cost-usd", type=float)
    p = sub.add_parser("prepare_data")
    src = p.add_mutually_exclusive_group(required=True)
    src.add_argument("--source-jsonl")
    src.add_argument("--hf-dataset")
    p.add_argument("--hf-config")
    p.add_argument("--hf-data-files", nargs="+")
    p.add_argument("--hf-shard-checksums")
    p.add_argument("--hf-local-shards")
    p.add_argument("--revision", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--max-tokens", type=int, default=50_000_000)
    p.add_argument("--max-documents", type=int, default=100_000)
    p.add_argument("--workers", type=int, default=1)
    p.add_argument("--tokenization-batch-bytes", type=int, default=1 << 20)
    p.add_argument("--exclude-validation-manifest")
    p = sub.add_parser("prepare_mechanisms")
    p.add_argument("--out", required=True)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--train-examples", type=int, default=32)
    p.add_argument("--validation-examples", type=int, default=16)
    p = sub.add_parser("evaluate_mechanisms")
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--task-manifest", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--max-examples", type=int, default=32)
    p.add_argument("--max-prompt-tokens", type=int)
    p.add_argument("--max-seconds", type=float, required=True)
    p.add_argument("--component", action="append")
    p.add_argument("--run-budget-usd", type=float)
    p.add_argument("--device", default="cpu")
    for name in ("train", "cooldown", "branch"):
        p = sub.add_parser(name)
        p.add_argument("--config", required=True)
        p.add_argument("--run-dir", required=True)
        p.add_argument("--max-steps", type=int, required=True)
        p.add_argument("--max-seconds", type=float, required=True)
        p.add_argument("--run-budget-usd", type=float)
        p.add_argument("--device", default="cuda")
        p.add_argument("--resume", required=name in ("cooldown", "branch"))
        p.add_argument("--context-fork", action="store_true")
        p.add_argument("--distributed", action="store_true", help="one process per GPU under torchrun")
        p.add_argument("--export-max-state-bytes", type=int)
        p.add_argument("--checkpoint-format", default="ttb-sharded-v1", choices=["ttb-sharded-v1", "tnlm-dcp-v1"],
                       help="format of --distributed recovery checkpoints (tnlm-dcp-v1: the reference's)")
        p.add_argument("--collective-timeout-seconds", type=float, default=120.0)
        if name == "branch":
            p.add_argument("--batch-tokens", type=int, required=True)
            p.add_argument("--lr-scale", type=float, required=True)
        if name == "cooldown":
            p.add_argument("--cooldown-steps", type=int, required=True)
            p.add_argument("--cooldown-end-tokens", type=int)
    p = sub.add_parser("profile")
    p.add_argument("--config", required=True)
    p.add_argument("--run-dir", required=True)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup-steps", type=int, default=2)
    p.add_argument("--kernels", action="store_true")
    p.add_argument("--trace-steps", type=int, default=0)
    p.add_argument("--max-seconds", type=float, required=True)
    p.add_argument("--run-budget-usd", type=float)
    p.add_argument("--device", default="cuda")
    p = sub.add_parser("analyze")
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--batches", type=int, default=2)
    p.add_argument("--rw-layer-window", type=int, metavar="K")
    p.add_argument("--context", type=int)
    p.add_argument("--max-seconds", type=float, default=300)
    p.add_argument("--run-budget-usd", type=float)
    p.add_argument("--device", default="cpu")
    p = sub.add_parser("evaluate")
    p.add_argument("--config", required=True)
    p.add_argument("--checkpoint", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--context", type=int)
    p.add_argument("--max-prediction-tokens", type=int, default=1_000_000)
    p.add_argument("--max-seconds", type=float, required=True)
    p.add_argument("--bootstrap-samples", type=int, default=1000)
    p.add_argument("--run-budget-usd", type=float)
    p.add_argument("--device", default="cpu")
    p = sub.add_parser("record_spend")
    p.add_argument("--config", required=True)
    p.add_argument("--charge-id", required=True)
    p.add_argument("--usd", type=float, required=True)
    p.add_argument("--stage", required=True, choices=("A", "B", "C", "D", "Reserve"))
    p.add_argument("--description", required=True)
    p = sub.add_parser("compare_evaluations")
    ci = p.add_mutually_exclusive_group(required=True)
    ci.add_argument("--left")
    ci.add_argument("--pairs")
    p.add_argument("--right")
    p.add_argument("--out", required=True)
    p.add_argument("--bootstrap-samples", type=int, default=1000)
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("compare_seed_pairs")
    p.add_argument("--pairs", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--allow-differences", nargs="*", default=[])
    p = sub.add_parser("summarize")
    p.add_argument("--run-dirs", nargs="+", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--max-plot-points", type=int, default=2000)
    p = sub.add_parser("check_math")
    p.add_argument("--verbose", action="store_true")
    return parser


def _sweep(cfg, args):
    import yaml

    from .sweep import run_sweep
    candidates = yaml.safe_load(Path(args.candidates).read_text())
    canary = args.canary_steps or args.min_tok_s is not None or args.canary_warmup_steps != 12
    preview = None
    if args.snapshot_sources is not None:
        from .search import plan_sweep
        planned = plan_sweep(cfg, candidates)
        policies = [r["config"].get("project", {}).get("dry_run", True) for r in planned["runs"]]
        if any(type(v) is not bool for v in policies) or len(set(policies)) != 1:
            raise ValueError("all candidates must share an explicit Boolean dry_run policy")
        snap = Path(args.snapshot_sources or (str(args.out) + ".sources")).absolute()
        preview = {"path": str(snap), "created": False,
                   "scope": "fresh source/config/grid snapshot; dependencies and data remain external"}
        if not policies[0]:
            from .source_snapshot import create_snapshot, run_snapshot
            if Path(args.out).exists() or Path(args.out).is_symlink():
                raise FileExistsError("automatic source snapshot requires a fresh sweep output")
            if snap.resolve().is_relative_to(Path(args.out).resolve()) or Path(args.out).resolve().is_relative_to(snap.resolve()):
                raise ValueError("source snapshot and sweep output directories must not overlap")
            config_path, cand_path = Path(args.config).resolve(), Path(args.candidates).resolve()
            create_snapshot(Path(__file__).resolve().parents[1], snap, inputs=[config_path, cand_path], workdir=Path.cwd())
            child = ["sweep", "--config", str(config_path), "--candidates", str(cand_path),
                     "--out", str(Path(args.out).absolute()), "--max-seconds", str(args.max_seconds),
                     "--evaluation-max-seconds", str(args.evaluation_max_seconds),
                     "--max-prediction-tokens", str(args.max_prediction_tokens),
                     "--bootstrap-samples", str(args.bootstrap_samples), "--device", args.device]
            if args.no_cooldown:
                child.append("--no-cooldown")
            if args.reference_candidate is not None:
                child += ["--reference-candidate", args.reference_candidate]
            if args.prune_completed_intermediates:
                child.append("--prune-completed-intermediates")
            if canary:
                child += ["--canary-steps", str(args.canary_steps), "--canary-warmup-steps", str(args.canary_warmup_steps)]
                if args.min_tok_s is not None:
                    child += ["--min-tok-s", str(args.min_tok_s)]
            return run_snapshot(snap, child, workdir=Path.cwd())
    result = run_sweep(cfg, candidates, args.out, max_seconds=args.max_seconds,
                       evaluation_max_seconds=args.evaluation_max_seconds, device=args.device,
                       cooldown=not args.no_cooldown, max_prediction_tokens=args.max_prediction_tokens,
                       bootstrap_samples=args.bootstrap_samples, reference_candidate=args.reference_candidate,
                       prune_completed_intermediates=args.prune_completed_intermediates,
                       **({"canary_steps": args.canary_steps, "min_tokens_per_second": args.min_tok_s,
                           "canary_warmup_steps": args.canary_warmup_steps} if canary else {}))
    if preview is not None:
        result["source_snapshot"] = preview
    return result


def main(argv=None):
    parser = _parser()
    args = parser.parse_args(argv)
    cmd = args.command
    result = None
    if cmd == "sweep-config":
        from .sweep_config import export_sweep_config
        text = export_sweep_config(args.sweep, args.candidate)
        if args.out is None:
            print(text, end="")
        else:
            with Path(args.out).open("x") as fh:
                fh.write(text)
        return 0
    if cmd == "compare_evaluations":
        if args.pairs is not None and args.right is not None:
            parser.error("--pairs cannot be combined with --right")
        if args.left is not None and args.right is None:
            parser.error("--left requires --right")
    if cmd == "reconcile":
        from .budget import SpendLedger
        ledger = SpendLedger(args.ledger)
        if args.apply:
            if not (args.expected_row_sha256 and args.operator and args.reason and args.all_workers_stopped):
                parser.error("--apply requires --expected-row-sha256, --operator, --reason and --all-workers-stopped")
            result = ledger.reconcile_terminal(args.run_id, expected_row_sha256=args.expected_row_sha256,
                                               operator=args.operator, reason=args.reason,
                                               terminal_attestation={"run_id": args.run_id, "all_workers_stopped": True},
                                               observed_elapsed_seconds=args.observed_elapsed_seconds,
                                               total_elapsed_seconds=args.total_elapsed_seconds,
                                               total_cost_usd=args.total_cost_usd, evidence_paths=args.metrics)
        else:
            if any(v is not None for v in (args.expected_row_sha256, args.operator, args.reason,
                                            args.observed_elapsed_seconds, args.total_elapsed_seconds,
                                            args.total_cost_usd)) or args.all_workers_stopped:
                parser.error("reconciliation controls require --apply")
            result = ledger.inspect_reconciliation(args.run_id, evidence_paths=args.metrics)
    elif cmd == "prepare_data":
        from .data import prepare_data
        kw = {}
        if args.hf_local_shards:
            kw["hf_local_shards"] = json.loads(Path(args.hf_local_shards).read_text())
        if args.hf_shard_checksums:
            kw["hf_shard_checksums"] = json.loads(Path(args.hf_shard_checksums).read_text())
        result = {"manifest": str(prepare_data(args.out, source_jsonl=args.source_jsonl, hf_dataset=args.hf_dataset,
                                               hf_config=args.hf_config, hf_data_files=args.hf_data_files,
                                               revision=args.revision, max_tokens=args.max_tokens,
                                               max_documents=args.max_documents, workers=args.workers,
                                               tokenization_batch_bytes=args.tokenization_batch_bytes,
                                               exclude_validation_manifest=args.exclude_validation_manifest, **kw))}
    elif cmd == "prepare_mechanisms":
        from .tasks import prepare_mechanism_tasks
        result = {"manifest": str(prepare_mechanism_tasks(args.out, seed=args.seed, train_examples=args.train_examples,
                                                          validation_examples=args.validation_examples))}
    elif cmd == "compare_evaluations":
        if args.pairs is not None:
            from .comparison_batch import compare_evaluation_pairs
            result = compare_evaluation_pairs(_pairs_file(args.pairs, ("left", "right")), args.out,
                                              bootstrap_samples=args.bootstrap_samples, seed=args.seed)
        else:
            from .evaluate import compare_evaluations
            result = compare_evaluations(args.left, args.right, args.out, bootstrap_samples=args.bootstrap_samples,
                                         seed=args.seed)
    elif cmd == "compare_seed_pairs":
        from .replication import compare_seed_pairs
        result = compare_seed_pairs(_pairs_file(args.pairs, ("left", "right")), args.out,
                                    allowed_between_dimensions=args.allow_differences)
    elif cmd == "summarize":
        from .reporting import summarize_runs
        result = summarize_runs(args.run_dirs, args.out, max_plot_points=args.max_plot_points)
    elif cmd == "check_math":
        import pytest
        tests = Path(__file__).resolve().parents[1] / "tests" / "test_math.py"
        return pytest.main([str(tests), "-v" if args.verbose else "-q"])
    else:
        cfg = Config.from_yaml(args.config)
        if cmd == "record_spend":
            from .budget import SpendLedger
            project = cfg.raw.get("project", {})
            if project.get("dry_run", True):
                result = {"dry_run": True, "charge_id": args.charge_id, "usd": args.usd, "stage": args.stage}
            else:
                ledger = SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                                     project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets"))
                result = ledger.record_charge(args.charge_id, args.usd, stage=args.stage, description=args.description)
        elif cmd == "validate_config":
            result = validate_config(cfg, device=args.device, run_dir=args.run_dir)
        elif cmd == "plan_search":
            if args.candidates:
                import yaml

                from .search import plan_sweep
                result = plan_sweep(cfg, yaml.safe_load(Path(args.candidates).read_text()))
            else:
                result = plan_search(cfg)
        elif cmd == "sweep":
            result = _sweep(cfg, args)
            if isinstance(result, int):
                return result
        elif cmd == "evaluate_mechanisms":
            from .evaluate import evaluate_mechanisms
            result = evaluate_mechanisms(cfg, args.checkpoint, args.task_manifest, args.out,
                                         max_examples=args.max_examples, max_prompt_tokens=args.max_prompt_tokens,
                                         max_seconds=args.max_seconds, device=args.device,
                                         components=tuple(args.component) if args.component else ("0:attn", "0:mlp"),
                                         run_budget_usd=args.run_budget_usd)
        elif cmd == "evaluate":
            from .evaluate import evaluate_checkpoint
            result = evaluate_checkpoint(cfg, args.checkpoint, args.out, context=args.context,
                                         max_prediction_tokens=args.max_prediction_tokens, max_seconds=args.max_seconds,
                                         device=args.device, bootstrap_samples=args.bootstrap_samples,
                                         run_budget_usd=args.run_budget_usd)
        elif cmd == "profile":
            result = profile_run(cfg, args.run_dir, steps=args.steps, warmup_steps=args.warmup_steps,
                                 max_seconds=args.max_seconds, device=args.device, run_budget_usd=args.run_budget_usd,
                                 kernels=args.kernels, trace_steps=args.trace_steps)
        elif cmd == "analyze":
            from .analysis import analyze_checkpoint
            result = analyze_checkpoint(cfg, args.checkpoint, args.out, batches=args.batches, context=args.context,
                                        max_seconds=args.max_seconds, device=args.device,
                                        run_budget_usd=args.run_budget_usd, rw_layer_window=args.rw_layer_window)
        elif cmd == "branch" and args.distributed:
            raise ValueError("batch branch supports serial training only")
        elif cmd in ("train", "cooldown") and args.distributed:
            result = _distributed_run(cfg, args)
        else:
            if args.export_max_state_bytes is not None:
                raise ValueError("--export-max-state-bytes is for --distributed; full-state checkpoints already evaluate")
            if args.checkpoint_format != "ttb-sharded-v1":
                raise ValueError("--checkpoint-format selects --distributed checkpoints; serial runs write full-state ones")
            result = train_run(cfg, args.run_dir, max_steps=args.max_steps, max_seconds=args.max_seconds,
                               device=args.device, resume=args.resume, run_budget_usd=args.run_budget_usd,
                               context_fork=args.context_fork, cooldown_steps=getattr(args, "cooldown_steps", None),
                               cooldown_end_tokens=getattr(args, "cooldown_end_tokens", None),
                               **({"batch_tokens": args.batch_tokens, "lr_scale": args.lr_scale}
                                  if cmd == "branch" else {}))
    if result is not None:
        print(json.dumps(result, indent=2, allow_nan=False, default=str))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
