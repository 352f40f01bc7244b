"""Checkpoint and numerics compatibility with the reference package (installed offline under
baseline/_ref; skipped where it is absent): state dicts load both ways and give the same logits."""
import os
import sys

import pytest
import torch

from helpers import TINY_MODEL

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def tnlm():
    if not os.path.isdir(os.path.join(REF, "tnlm")):
        pytest.skip("reference package not installed")
    sys.path.insert(0, REF)
    try:
        import tnlm.checkpoint
        import tnlm.config
        import tnlm.model
        import tnlm.optim
        yield tnlm
    finally:
        sys.path.remove(REF)


@pytest.mark.parametrize("normalization", ["pre_rms", "group_rms", "sandwich_rms", "spectral_rms"])
@pytest.mark.parametrize("attention", ["signed_product", "offset_square", "lower_degree_mix"])
def test_reference_checkpoint_loads_with_identical_logits(tnlm, tmp_path, normalization, attention):
    from tensor_train_ing_b200.checkpoint import load_checkpoint
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    kw = dict(TINY_MODEL, normalization=normalization, attention=attention)
    torch.manual_seed(3)
    ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**kw)).double().eval()
    tnlm.checkpoint.save_checkpoint(tmp_path / "ck", ref, None, None, config={"model": kw}, progress={"steps": 0},
                                    manifest_hash="0" * 64)
    ours = TensorLM(ModelConfig(**kw)).double().eval()
    load_checkpoint(tmp_path / "ck", ours, restore_rng=False)
    idx = torch.randint(0, 97, (2, 11))
    doc = torch.tensor([[0] * 6 + [1] * 5, [0] * 11])
    with torch.no_grad():
        a = ref(idx, doc_ids=doc)
        b = ours(idx, doc_ids=doc)
    torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-10)


def test_our_checkpoint_loads_in_reference(tnlm, tmp_path):
    from tensor_train_ing_b200.checkpoint import save_checkpoint
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    torch.manual_seed(4)
    ours = TensorLM(ModelConfig(**TINY_MODEL)).eval()
    save_checkpoint(tmp_path / "ck", ours, None, None, config={"model": TINY_MODEL}, progress={"steps": 0},
                    manifest_hash="0" * 64)
    ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**TINY_MODEL)).eval()
    tnlm.checkpoint.load_checkpoint(tmp_path / "ck", ref, restore_rng=False)
    idx = torch.randint(0, 97, (1, 9))
    with torch.no_grad():
        torch.testing.assert_close(ref(idx), ours(idx))


def test_same_seed_same_initialisation(tnlm):
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    torch.manual_seed(11)
    ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**TINY_MODEL))
    torch.manual_seed(11)
    ours = TensorLM(ModelConfig(**TINY_MODEL))
    rs, os_ = ref.state_dict(), ours.state_dict()
    assert rs.keys() == os_.keys()
    for k in rs:
        assert torch.equal(rs[k], os_[k]), k


def _dataset(tmp_path, n=120):
    import json
    import random

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.data import prepare_data
    rnd = random.Random(0)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"d{i}", "text": "".join(rnd.choice("abcdefgh ")
                                                                         for _ in range(rnd.randint(3, 90)))}) + "\n"
                           for i in range(n)))
    return prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                        split_fractions={"train": .8, "val": .1, "test": 0., "calibration": .1})


def test_datasets_sampler_index_and_batches_are_shared_with_the_reference(tnlm, tmp_path):
    """A dataset prepared here, with the sampler index built here, is accepted by the reference's
    verifier, and both frameworks' packed samplers (and rank samplers) yield identical batches."""
    import shutil

    import tnlm.data as ref_data

    from tensor_train_ing_b200.data import PackedSampler, RankPackedSampler
    from tensor_train_ing_b200.sampler_index import INDEX_DIR
    manifest = _dataset(tmp_path)
    for split in ("train", "val", "calibration"):
        for ctx, rows, seed in ((16, 4, 0), (33, 3, 7)):
            ours = PackedSampler(manifest, split=split, batch_size=rows, context=ctx, seed=seed)
            theirs = ref_data.PackedSampler(manifest, split=split, batch_size=rows, context=ctx, seed=seed)
            for _ in range(25):
                for a, b in zip(ours.next_batch(), theirs.next_batch()):
                    assert torch.equal(a, b)
    for r in range(3):
        ours = RankPackedSampler(manifest, rank=r, world_size=3, batch_size=2, context=16, seed=5)
        theirs = ref_data.RankPackedSampler(manifest, rank=r, world_size=3, batch_size=2, context=16, seed=5)
        for _ in range(10):
            for a, b in zip(ours.next_batch(), theirs.next_batch()):
                assert torch.equal(a, b)
    # an index the reference built is accepted here without a rebuild
    root = manifest.parent
    shutil.rmtree(root / INDEX_DIR)
    ref_data.PackedSampler(manifest, split="train", batch_size=1, context=16, seed=0)
    built = {p.name: p.stat().st_mtime_ns for p in (root / INDEX_DIR).iterdir()}
    PackedSampler(manifest, split="train", batch_size=1, context=16, seed=0)
    assert {p.name: p.stat().st_mtime_ns for p in (root / INDEX_DIR).iterdir()} == built


def test_the_same_source_prepares_byte_identical_datasets(tnlm, tmp_path):
    """Dataset preparation here and in the reference give the same bytes for every artifact, so the
    manifest sha256 (the dataset identity that checkpoints and resumes compare) is shared."""
    import json
    import random

    import tnlm.data as ref_data

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.data import prepare_data
    rnd = random.Random(3)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"d{i}", "text": "".join(rnd.choice("abc\r\n xyz")
                                                                         for _ in range(rnd.randint(1, 80)))}) + "\n"
                           for i in range(90)))
    kw = dict(source_jsonl=src, revision="offline-v1", max_documents=70,
              split_fractions={"train": .7, "val": .1, "test": .1, "calibration": .1})
    prepare_data(tmp_path / "ours", tokenizer=FixtureTokenizer(), **kw)
    ref_data.prepare_data(tmp_path / "ref", tokenizer=FixtureTokenizer(), **kw)
    names = sorted(p.name for p in (tmp_path / "ours").iterdir() if p.is_file())
    assert "manifest.json" in names and "documents.jsonl" in names
    for name in names:
        assert (tmp_path / "ours" / name).read_bytes() == (tmp_path / "ref" / name).read_bytes(), name


def test_schedules_and_optimizer_updates_match_the_reference(tnlm):
    import tnlm.schedules as ref_sched

    from tensor_train_ing_b200 import schedules
    from tensor_train_ing_b200.config import ModelConfig, TrainConfig
    from tensor_train_ing_b200.models.model import TensorLM
    from tensor_train_ing_b200.optim import make_optimizer
    def outcome(fn, *args, **kwargs):  # the value, or the exception type (short cosine horizons are refused)
        try:
            return fn(*args, **kwargs)
        except Exception as e:  # noqa: BLE001
            return type(e).__name__

    for total in (1, 7, 150, 1000, 12345):
        for kind in ("constant_with_separate_cooldown", "cosine"):
            for step in sorted({0, 1, 2, total // 3, max(0, total - 2), total - 1, total, total + 5}):
                assert outcome(schedules.schedule_multiplier, step, total, schedule=kind) == \
                    outcome(ref_sched.schedule_multiplier, step, total, schedule=kind), (total, kind, step)
    mk = dict(layers=2, d_model=16, heads=2, d_key=8, d_value=8, d_mlp=24, vocab_size=40, padded_vocab=64)
    for opt in ("adamw", "muon"):
        tk = dict(optimizer=opt, lr=1e-2, aux_adamw_lr=3e-3, compile=False, bf16_compute=False)
        torch.manual_seed(0)
        ours = TensorLM(ModelConfig(**mk))
        ref = tnlm.model.TensorLM(tnlm.config.ModelConfig(**mk))
        ref.load_state_dict(ours.state_dict())
        o_ours, o_ref = make_optimizer(ours, TrainConfig(**tk)), tnlm.optim.make_optimizer(ref, tnlm.config.TrainConfig(**tk))
        for step in range(3):
            g = torch.Generator().manual_seed(step)
            grads = {k: torch.randn(p.shape, generator=g) * 0.01 for k, p in ours.named_parameters()}
            for model in (ours, ref):
                for k, p in model.named_parameters():
                    p.grad = grads[k].clone()
            o_ours.step()
            o_ref.step()
        ref_params = dict(ref.named_parameters())
        for k, p in ours.named_parameters():
            assert torch.equal(p, ref_params[k]), (opt, k)  # bit-identical updates


@pytest.mark.parametrize("optimizer,normalization", [("adamw", "pre_rms"), ("muon", "pre_rms"),
                                                     ("muon", "group_rms"), ("adamw", "lagged")])
def test_serial_training_trajectories_match_the_reference(tnlm, tmp_path, optimizer, normalization):
    """Both frameworks' serial trainers on one YAML config and dataset (CPU): identical per-step losses
    and identical final weights (lagged norms include the calibration before the first update)."""
    import json

    import tnlm.train as ref_train
    import yaml

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    model = {"layers": 2, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12, "padded_vocab": 50257,
             "normalization": normalization}
    if normalization == "lagged":
        model["final_normalization"] = "lagged"
    runs = {}
    for who, run in (("ours", train_run), ("reference", ref_train.train_run)):
        doc = {"model": model,
               "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                         "rung_total_tokens": 200, "lr": 0.01, "optimizer": optimizer, "aux_adamw_lr": 0.003},
               "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2, "calibration_tokens": 8},
               "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / f"{who}.json")}}
        path = tmp_path / f"{who}.yaml"
        path.write_text(yaml.safe_dump(doc))
        cfg = Config.from_yaml(str(path)) if who == "ours" else tnlm.config.Config.from_yaml(str(path))
        result = run(cfg, tmp_path / who, max_steps=5, max_seconds=120, device="cpu")
        losses = [json.loads(l)["loss"] for l in (tmp_path / who / "metrics.jsonl").read_text().splitlines()]
        runs[who] = (losses, result["checkpoint"])
    assert len(runs["ours"][0]) == 5 and runs["ours"][0] == runs["reference"][0]
    ours = torch.load(f"{runs['ours'][1]}/state.pt", weights_only=False)["model"]
    theirs = torch.load(f"{runs['reference'][1]}/state.pt", weights_only=False)["model"]
    assert ours.keys() == theirs.keys()
    for k in ours:
        assert torch.equal(ours[k], theirs[k]), k


def test_evaluation_reports_agree_and_cross_compare_with_the_reference(tnlm, tmp_path):
    """One checkpoint evaluated by both frameworks: identical held-out CE and per-document losses, and
    each framework's paired comparator accepts the other's report (provenance fields differ)."""
    import json

    import tnlm.evaluate as ref_eval
    import yaml

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.evaluate import compare_evaluations, evaluate_checkpoint
    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    doc = {"model": {"layers": 2, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json")}}
    path = tmp_path / "run.yaml"
    path.write_text(yaml.safe_dump(doc))
    ckpt = train_run(Config.from_yaml(str(path)), tmp_path / "run", max_steps=3, max_seconds=120,
                     device="cpu")["checkpoint"]
    ours = evaluate_checkpoint(Config.from_yaml(str(path)), ckpt, tmp_path / "ours", max_seconds=120,
                               bootstrap_samples=20)
    theirs = ref_eval.evaluate_checkpoint(tnlm.config.Config.from_yaml(str(path)), ckpt, tmp_path / "ref",
                                          max_seconds=120, bootstrap_samples=20)
    assert ours["ce"] == theirs["ce"] and ours["prediction_tokens"] == theirs["prediction_tokens"]
    assert ours["per_document"] == theirs["per_document"]
    a, b = tmp_path / "ours" / "evaluation.json", tmp_path / "ref" / "evaluation.json"
    for compare in (compare_evaluations, ref_eval.compare_evaluations):
        for left, right in ((a, b), (b, a)):
            assert compare(left, right, None, bootstrap_samples=10)["delta_ce_right_minus_left"] == 0.0


def test_mechanism_task_sets_are_byte_identical_to_the_reference(tnlm, tmp_path):
    import tnlm.tasks as ref_tasks

    from tensor_train_ing_b200.tasks import prepare_mechanism_tasks
    for seed, train, val in ((0, 8, 8), (7, 32, 16)):
        prepare_mechanism_tasks(tmp_path / f"ours{seed}", seed=seed, train_examples=train, validation_examples=val)
        ref_tasks.prepare_mechanism_tasks(tmp_path / f"ref{seed}", seed=seed, train_examples=train,
                                          validation_examples=val)
        names = sorted(p.name for p in (tmp_path / f"ours{seed}").iterdir() if p.is_file())
        assert names == sorted(p.name for p in (tmp_path / f"ref{seed}").iterdir() if p.is_file())
        for name in names:
            assert (tmp_path / f"ours{seed}" / name).read_bytes() == (tmp_path / f"ref{seed}" / name).read_bytes()


def test_run_summaries_read_reference_run_directories(tnlm, tmp_path):
    """`summarize` over one run of each framework (same config and data): the reference's result.json,
    metrics and ledger are read like ours, and every non-timing field of the two rows agrees."""
    import json

    import tnlm.train as ref_train
    import yaml

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.reporting import summarize_runs
    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    doc = {"model": {"layers": 2, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json")}}
    path = tmp_path / "run.yaml"
    path.write_text(yaml.safe_dump(doc))
    train_run(Config.from_yaml(str(path)), tmp_path / "ours", max_steps=3, max_seconds=120, device="cpu")
    ref_train.train_run(tnlm.config.Config.from_yaml(str(path)), tmp_path / "ref", max_steps=3, max_seconds=120,
                        device="cpu")
    out = summarize_runs([tmp_path / "ours", tmp_path / "ref"], tmp_path / "summary")
    assert out["runs"] == 2
    rows = json.loads((tmp_path / "summary" / "comparison.json").read_text())["runs"]
    timing = {"run", "run_elapsed_seconds", "run_billed_usd", "step_average_prediction_tokens_per_second",
              "cuda_peak_allocated_bytes", "cuda_peak_reserved_bytes"}
    assert {k: v for k, v in rows[0].items() if k not in timing} == {k: v for k, v in rows[1].items()
                                                                    if k not in timing}


@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
def test_a_reference_run_resumed_here_continues_exactly(tnlm, tmp_path, optimizer):
    """3 steps in the reference trainer, then 2 more here from its checkpoint (model, optimizer,
    sampler cursor, RNG): the losses and final weights equal those of one uninterrupted 5-step
    reference run, so a run can switch frameworks mid-way."""
    import json

    import tnlm.train as ref_train
    import yaml

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    doc = {"model": {"layers": 2, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01, "optimizer": optimizer, "aux_adamw_lr": 0.003},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json")}}
    path = tmp_path / "run.yaml"
    path.write_text(yaml.safe_dump(doc))
    ref_cfg = lambda: tnlm.config.Config.from_yaml(str(path))  # noqa: E731
    full = ref_train.train_run(ref_cfg(), tmp_path / "full", max_steps=5, max_seconds=120, device="cpu")
    first = ref_train.train_run(ref_cfg(), tmp_path / "first", max_steps=3, max_seconds=120, device="cpu")
    rest = train_run(Config.from_yaml(str(path)), tmp_path / "rest", max_steps=2, max_seconds=120, device="cpu",
                     resume=first["checkpoint"])
    losses = lambda d: [json.loads(l)["loss"] for l in (tmp_path / d / "metrics.jsonl").read_text().splitlines()]  # noqa: E731
    assert losses("full") == losses("first") + losses("rest")
    a = torch.load(f"{full['checkpoint']}/state.pt", weights_only=False)["model"]
    b = torch.load(f"{rest['checkpoint']}/state.pt", weights_only=False)["model"]
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
def test_a_run_from_here_resumed_by_the_reference_continues_exactly(tnlm, tmp_path, optimizer):
    """The reverse direction: 3 steps here, 2 more in the reference trainer from our checkpoint, equal
    to an uninterrupted 5-step run here (our Muon checkpoints carry the reference's optimizer identity,
    which its loader requires)."""
    import json

    import tnlm.train as ref_train
    import yaml

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    doc = {"model": {"layers": 2, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01, "optimizer": optimizer, "aux_adamw_lr": 0.003},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json")}}
    path = tmp_path / "run.yaml"
    path.write_text(yaml.safe_dump(doc))
    full = train_run(Config.from_yaml(str(path)), tmp_path / "full", max_steps=5, max_seconds=120, device="cpu")
    first = train_run(Config.from_yaml(str(path)), tmp_path / "first", max_steps=3, max_seconds=120, device="cpu")
    rest = ref_train.train_run(tnlm.config.Config.from_yaml(str(path)), tmp_path / "rest", max_steps=2,
                               max_seconds=120, device="cpu", resume=first["checkpoint"])
    losses = lambda d: [json.loads(l)["loss"] for l in (tmp_path / d / "metrics.jsonl").read_text().splitlines()]  # noqa: E731
    assert losses("full") == losses("first") + losses("rest")
    a = torch.load(f"{full['checkpoint']}/state.pt", weights_only=False)["model"]
    b = torch.load(f"{rest['checkpoint']}/state.pt", weights_only=False)["model"]
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


def test_checkpoint_storage_plans_match_the_reference(tnlm):
    """Milestones, retention and the disk forecast agree field for field (the reference adds a descriptive
    `assumptions` list, partly about its DCP layout, which this plan does not carry)."""
    import tnlm.checkpoint_plan as ref_plan

    from tensor_train_ing_b200 import checkpoint_plan
    from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
    mk = dict(layers=4, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=768)
    for optimizer in ("adamw", "muon"):
        for rung, batch in ((10_000_000, 8192), (2_000_000_000, 524288)):
            tk = dict(optimizer=optimizer, rung_total_tokens=rung, global_prediction_tokens_per_update=batch)
            ours = checkpoint_plan.checkpoint_storage_plan(Config(model=ModelConfig(**mk), train=TrainConfig(**tk)))
            theirs = ref_plan.checkpoint_storage_plan(tnlm.config.Config(model=tnlm.config.ModelConfig(**mk),
                                                                         train=tnlm.config.TrainConfig(**tk)))
            assert set(theirs) - set(ours) == {"assumptions"} and not set(ours) - set(theirs)
            assert all(ours[k] == theirs[k] for k in ours), (optimizer, rung)


@pytest.mark.parametrize("case", [
    dict(plan=dict(token_limit=10_000_000, max_steps=2)),
    dict(plan=dict(token_limit=1_000_000_000, distributed=True, distributed_world_size=2)),
    dict(plan=dict(token_limit=10_000_000, cooldown=True)),
    dict(plan=dict(start_tokens=2_000_000, token_limit=4_000_001, max_steps=1)),
    dict(plan=dict(max_steps=0, export_weights=True)),
    dict(plan=dict(token_limit=10 ** 40)),
    dict(plan=dict(max_steps=0, export_weights=True, distributed=True, distributed_world_size=3), tie=True),
    dict(plan=dict(token_limit=16), milestones=[7, 14, 14]),
    dict(plan=dict(token_limit=20_000_000, distributed=True, distributed_world_size=2), milestones=[]),
    dict(plan=dict(max_steps=0), normalization="spectral_rms", optimizer="muon"),
    dict(plan=dict(token_limit=200_000_000, max_steps=123), retention=dict(keep_recovery_checkpoints=0,
                                                                            save_initial_checkpoint=False)),
])
def test_checkpoint_storage_plan_edge_cases_match_the_reference(tnlm, case):
    """Resumes, zero-update runs, horizons beyond any int64, tied embeddings, explicit and empty
    milestone lists, the cooldown and distributed branch rules and the retention switches give the
    reference's plan field for field."""
    import tnlm.checkpoint_plan as ref_plan

    from tensor_train_ing_b200 import checkpoint_plan
    from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
    mk = dict(layers=1, d_model=8, heads=1, d_key=4, d_value=4, d_mlp=12, vocab_size=16, padded_vocab=16,
              attention_backend="reference", tie_embeddings=case.get("tie", False),
              normalization=case.get("normalization", "pre_rms"))
    tk = dict(global_prediction_tokens_per_update=1_000_000, optimizer=case.get("optimizer", "adamw"))
    project = {}
    if "milestones" in case:
        project["milestone_tokens"] = case["milestones"]
    project.update(case.get("retention", {}))
    ours = checkpoint_plan.checkpoint_storage_plan(
        Config(model=ModelConfig(**mk), train=TrainConfig(**tk), raw={"project": dict(project)}), **case["plan"])
    theirs = ref_plan.checkpoint_storage_plan(
        tnlm.config.Config(model=tnlm.config.ModelConfig(**mk), train=tnlm.config.TrainConfig(**tk),
                           raw={"project": dict(project)}), **case["plan"])
    theirs.pop("assumptions")
    assert ours == theirs


def test_training_evidence_descriptors_match_the_reference(tnlm):
    """The training evidence an evaluation report carries (batch and context histories, cooldown and
    completion status) is the reference's, field for field, on valid, partial, malformed and
    inconsistent checkpoint payloads, and so are the comparisons built from it."""
    import copy
    import itertools

    import tnlm.evaluate as ref_eval

    from tensor_train_ing_b200 import evaluate as our_eval
    base = {"config": {"train": {"global_prediction_tokens_per_update": 48, "lr": 0.03, "aux_adamw_lr": None,
                                 "rung_total_tokens": 480, "schedule": "constant"},
                       "model": {"d_model": 64, "layers": 2}, "data": {"context": 32}},
            "progress": {"tokens": 160, "steps": 6, "scheduler_step": 6, "batch_history": [
                {"batch_tokens": 16, "lr": 0.01, "aux_adamw_lr": None, "start_tokens": 0, "start_step": 0,
                 "source": "fresh"},
                {"batch_tokens": 48, "lr": 0.03, "aux_adamw_lr": None, "start_tokens": 64, "start_step": 4,
                 "source": "batch_branch", "lr_scale": 3.0, "parent": {"path": "/p"}}],
                "context_history": [{"context": 16, "start_tokens": 0, "start_step": 0, "source": "fresh"},
                                    {"context": 32, "start_tokens": 96, "start_step": 5, "source": "context_fork"}]},
            "extra": {"cooldown_steps": None}}
    edits = [None, ("batch_history", 0, "source", "legacy_unknown"), ("batch_history", 1, "start_tokens", 161),
             ("batch_history", 1, "lr_scale", 0), ("batch_history", 1, "lr", 0.05),
             ("batch_history", 0, "batch_tokens", True), ("context_history", 1, "context", 8),
             ("context_history", 1, "source", "fresh"), ("context_history", 0, "source", "legacy_unknown"),
             ("context_history", 1, "start_step", 9), ("extra", None, "cooldown_steps", 4),
             ("progress", None, "cooldown_start_tokens", 120), ("progress", None, "tokens", 480),
             ("config", "train", "schedule", "cosine")]
    # combinations that reach the cooldown endpoint and completion rules
    cooled = [("extra", None, "cooldown_steps", 2), ("progress", None, "cooldown_start_tokens", 96)]
    edits += [tuple(cooled),
              tuple(cooled + [("progress", None, "cooldown_end_tokens", 190)]),   # inside the last update
              tuple(cooled + [("progress", None, "cooldown_end_tokens", 140)]),   # before it: refused
              tuple(cooled + [("progress", None, "tokens", 192), ("progress", None, "scheduler_step", 2)]),
              tuple(cooled + [("progress", None, "tokens", 192), ("progress", None, "scheduler_step", 1)]),
              tuple(cooled + [("progress", None, "distributed_schedule", {"cooldown_steps": 3})]),
              (("extra", None, "cooldown_steps", 0),),
              (("config", "train", "schedule", "cosine"), ("progress", None, "tokens", 480),
               ("progress", None, "scheduler_step", 10)),
              (("config", "train", "schedule", "cosine"), ("progress", None, "scheduler_step", 11))]

    def apply(p, edit):
        where, i, field, value = edit
        if where in ("batch_history", "context_history"):
            p["progress"][where][i][field] = value
        elif where == "config":
            p["config"][i][field] = value
        else:
            p[where][field] = value
    payloads = []
    for edit in edits:
        p = copy.deepcopy(base)
        for one in (() if edit is None else edit if isinstance(edit[0], tuple) else (edit,)):
            apply(p, one)
        payloads.append(p)
    ours = [our_eval._training_descriptor(p) for p in payloads]
    # the reference adds two descriptive sentences about the histories' scope; the values are compared
    theirs = [{k: v for k, v in ref_eval._training_descriptor(p).items()
               if k not in ("batch_history_scope", "context_history_scope")} for p in payloads]
    for o, t, edit in zip(ours, theirs, edits):
        assert o == t, edit
    for a, b in itertools.combinations(range(len(payloads)), 2):
        mine = our_eval._training_comparison({"training_descriptor": ours[a]}, {"training_descriptor": ours[b]})
        ref = ref_eval._training_comparison({"training_descriptor": theirs[a]}, {"training_descriptor": theirs[b]})
        mine.pop("scope"), ref.pop("scope")  # descriptive sentences
        assert mine == ref, (edits[a], edits[b])


@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
def test_optimizer_exposure_records_match_the_reference(tnlm, optimizer):
    """The exposure record a checkpoint carries (group identities and digests, rate and decay sums,
    the shrinkage product with zero and negative factors) is the reference's after the same updates."""
    import json

    import tnlm.optimizer_exposure as ref_exposure

    from tensor_train_ing_b200.config import ModelConfig, TrainConfig
    from tensor_train_ing_b200.models.model import TensorLM
    from tensor_train_ing_b200.optim import make_optimizer
    from tensor_train_ing_b200.optimizer_exposure import update_optimizer_exposure
    tk = dict(optimizer=optimizer, lr=0.02, aux_adamw_lr=0.003, weight_decay_hidden=0.1)
    ours_opt = make_optimizer(TensorLM(ModelConfig(**TINY_MODEL)), TrainConfig(**tk))
    ref_opt = tnlm.optim.make_optimizer(tnlm.model.TensorLM(tnlm.config.ModelConfig(**TINY_MODEL)),
                                        tnlm.config.TrainConfig(**tk))
    progress = {"ours": {"steps": 3, "tokens": 30}, "ref": {"steps": 3, "tokens": 30}}
    for scale in (1.0, 0.0, 50.0, 60.0):  # ordinary, zero rate, lr * wd = 1 and above it
        for opt in (ours_opt, ref_opt):
            groups = (opt.muon.param_groups + opt.adamw.param_groups) if hasattr(opt, "muon") else opt.param_groups
            for g in groups:
                g["lr"] = 0.02 * scale
        update_optimizer_exposure(progress["ours"], ours_opt)
        ref_exposure.update_optimizer_exposure(progress["ref"], ref_opt)
        for side in progress.values():
            side["steps"] += 1
    ours, ref = (json.dumps(progress[k]["optimizer_exposure"], sort_keys=True) for k in ("ours", "ref"))
    assert ours == ref


def test_both_trainers_share_one_spend_ledger(tnlm, tmp_path):
    """Runs of either framework reserve, bill and complete entries in the same locked ledger file."""
    import json

    import tnlm.train as ref_train
    import yaml

    from helpers import FixtureTokenizer
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.data import prepare_data
    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    ledger = tmp_path / "shared-ledger.json"
    doc = {"model": {"layers": 1, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(ledger)}}
    path = tmp_path / "run.yaml"
    path.write_text(yaml.safe_dump(doc))
    train_run(Config.from_yaml(str(path)), tmp_path / "a", max_steps=2, max_seconds=60, device="cpu")
    ref_train.train_run(tnlm.config.Config.from_yaml(str(path)), tmp_path / "b", max_steps=2, max_seconds=60,
                        device="cpu")
    train_run(Config.from_yaml(str(path)), tmp_path / "c", max_steps=2, max_seconds=60, device="cpu")
    runs = json.loads(ledger.read_text())["runs"]
    assert len(runs) == 3 and all(r["status"] == "complete" for r in runs.values())
